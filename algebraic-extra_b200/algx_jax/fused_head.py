"""``fused_head`` for JAX over libalgx (drop-in for kernels/fused_head.py:260-275).

Same signature and ``custom_vjp`` residuals as the reference (h, E, targets,
stat; fused_head.py:240-254); the telemetry carries no gradient. The
objective and its statistics come from the XLA FFI target ``algx_head_fwd``,
dh and dE from ``algx_head_bwd``; ``ignore_index`` is this build's opt-in
extension (default None reproduces the reference).
"""

from __future__ import annotations

import functools

import jax
import jax.numpy as jnp
import numpy as np

from algx import variants as VA

from . import _ffi

_INT_ATTRS = ("kind", "n", "has_ignore", "ignore_index")
_FLOAT_ATTRS = ("inv_c", "clamp")


def _attrs(ints, floats):
    a = {name: np.int32(v) for name, v in zip(_INT_ATTRS, ints)}
    a.update({name: np.float32(v) for name, v in zip(_FLOAT_ATTRS, floats)})
    return a


def _fwd_call(h, e, t, ints, floats):
    core = _ffi.core()
    N, V = h.shape[0], e.shape[0]
    splits = int(core.algx_head_fwd_splits(N, V))
    f32 = jnp.float32
    obj, tel, stat, count, _, _ = jax.ffi.ffi_call(
        "algx_head_fwd",
        (jax.ShapeDtypeStruct((1,), f32), jax.ShapeDtypeStruct((N,), f32), jax.ShapeDtypeStruct((N,), f32),
         jax.ShapeDtypeStruct((1,), f32), jax.ShapeDtypeStruct((3 * splits * N,), f32),
         jax.ShapeDtypeStruct((3 * N,), f32)))(h, e, t, **_attrs(ints, floats))
    return obj, tel, stat, count


@functools.partial(jax.custom_vjp, nondiff_argnums=(3, 4, 5))
def _head(h, e, t, ints, floats, slope):
    obj, tel, _, _ = _fwd_call(h, e, t, ints, floats)
    return obj[0], tel


def _head_fwd(h, e, t, ints, floats, slope):
    obj, tel, stat, count = _fwd_call(h, e, t, ints, floats)
    return (obj[0], tel), (h, e, t, stat, count)


def _head_bwd(ints, floats, slope, res, g):
    h, e, t, stat, count = res
    g_obj, _ = g  # the telemetry is stop-gradient'ed by the caller
    N, d = h.shape
    V = e.shape[0]
    scale = (jnp.reshape(g_obj, (1,)).astype(jnp.float32) * slope / count).astype(jnp.float32)
    code = VA.ALGX_BF16 if h.dtype == jnp.bfloat16 else VA.ALGX_F32
    ws = max(int(_ffi.core().algx_head_bwd_workspace_size(N, d, V, code)), 1)
    dh, de, _ = jax.ffi.ffi_call(
        "algx_head_bwd",
        (jax.ShapeDtypeStruct(h.shape, h.dtype), jax.ShapeDtypeStruct(e.shape, jnp.float32),
         jax.ShapeDtypeStruct((ws,), jnp.uint8)))(h, e, t, stat, scale, **_attrs(ints, floats))
    return dh, de.astype(e.dtype), None


_head.defvjp(_head_fwd, _head_bwd)


def fused_head(h, embed, targets, *, kind="ce", n=16, c=16.0, block_n=128, block_v=512, ignore_index=None):
    """Fused tied-embedding projection and likelihood objective; returns
    ``(objective, telemetry)`` (kernels/fused_head.py:260-275)."""
    N, d = VA.check_head_options(kind, n, h.shape, block_n)
    if embed.shape[1] != d or targets.shape != (N,):
        raise ValueError("h (N, d), embed (V, d) and targets (N,) shapes disagree")
    ints, floats = VA.head_config_lists(kind, n, c, embed.shape[0], ignore_index)
    # the tensor-core GEMMs take bfloat16 operands (embed.astype(h.dtype), fused_head.py:168)
    h16 = h.astype(jnp.bfloat16)
    e16 = embed.astype(jnp.bfloat16)
    obj, tel = _head(h16, e16, targets.astype(jnp.int32), tuple(ints), tuple(floats), VA.head_slope(kind, n, c))
    return obj, jax.lax.stop_gradient(tel)
