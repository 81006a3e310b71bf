"""``flash_attention`` for JAX over libalgx (drop-in for kernels/flash.py:763-857).

Same signature, option checks (algx.variants) and ``custom_vjp`` residuals as
the reference (q_scaled, k, v, sink, O, stat; flash.py:713-726). The range
guard is decided on the device (no ``lax.cond``); the forward and backward
launch groups are the XLA FFI targets ``algx_attn_fwd`` and ``algx_attn_bwd``.
"""

from __future__ import annotations

import functools
from typing import Optional

import jax
import jax.numpy as jnp
import numpy as np

from algx import variants as VA

from . import _ffi

_INT_ATTRS = ("kind", "mode", "n", "fast_rho", "inv_stat", "has_sink")
_FLOAT_ATTRS = ("clamp", "scale", "guard_qk", "guard_sink", "guard_v")


def _attrs(ints, floats):
    a = {name: np.int32(v) for name, v in zip(_INT_ATTRS, ints)}
    a.update({name: np.float32(v) for name, v in zip(_FLOAT_ATTRS, floats)})
    return a


def _fwd_call(q, k, v, sink, ints, floats):
    _ffi.libs()
    B, H, T, D = q.shape
    guarded = ints[0] == VA.ALGX_ATTN_ASINH and ints[1] == VA.ALGX_MODE_GUARDED
    f32 = jnp.float32
    return jax.ffi.ffi_call(
        "algx_attn_fwd",
        (jax.ShapeDtypeStruct(q.shape, q.dtype),                            # o
         jax.ShapeDtypeStruct((B, H, T, D) if guarded else (0,), f32),      # o_precise
         jax.ShapeDtypeStruct((B, H, T), f32),                              # stat
         jax.ShapeDtypeStruct(q.shape, q.dtype),                            # q_scaled
         jax.ShapeDtypeStruct((4,), f32)))(q, k, v, sink, **_attrs(ints, floats))  # guard maxima


@functools.partial(jax.custom_vjp, nondiff_argnums=(4, 5))
def _flash(q, k, v, sink, ints, floats):
    return _fwd_call(q, k, v, sink, ints, floats)[0]


def _flash_fwd(q, k, v, sink, ints, floats):
    o, o_prec, stat, q_s, guard = _fwd_call(q, k, v, sink, ints, floats)
    return o, (q_s, k, v, sink, guard, o, o_prec, stat)


def _flash_bwd(ints, floats, res, do):
    q_s, k, v, sink, guard, o, o_prec, stat = res
    B, H, T, D = q_s.shape
    ws = max(int(_ffi.core().algx_attn_bwd_workspace_size(B, H, T, D)), 1)
    dq, dk, dv, dsink, _ = jax.ffi.ffi_call(
        "algx_attn_bwd",
        (jax.ShapeDtypeStruct(q_s.shape, q_s.dtype), jax.ShapeDtypeStruct(k.shape, k.dtype),
         jax.ShapeDtypeStruct(v.shape, v.dtype), jax.ShapeDtypeStruct(sink.shape, jnp.float32),
         jax.ShapeDtypeStruct((ws,), jnp.uint8)))(q_s, k, v, sink, guard, o, o_prec, stat, do.astype(q_s.dtype),
                                                 **_attrs(ints, floats))
    return dq, dk, dv, dsink


_flash.defvjp(_flash_fwd, _flash_bwd)


def flash_attention(q, k, v, sink_logit=None, *, kind: str = "softmax",
                    n: int = 16, c: float = 16.0, block: int = 512,
                    block_q: Optional[int] = None, block_k: Optional[int] = None,
                    shift: Optional[bool] = None, fast_rho: Optional[bool] = None,
                    inv_stat: Optional[bool] = None, compact_stat: bool = True,
                    poly_rho: bool = False, range_guard: bool = False,
                    resident_bwd: Optional[bool] = None,
                    diagonal_bwd: Optional[bool] = None,
                    diagonal_fwd: Optional[bool] = None,
                    head_resident: Optional[bool] = None):
    """Causal attention on (B, H, T, D); ``sink_logit`` broadcastable to (H,)
    (kernels/flash.py:763-857). D must be 64; q, k, v bfloat16 or float32."""
    B, H, T, D = q.shape
    var = VA.check_flash_options(T, D, q.dtype == k.dtype == v.dtype == jnp.bfloat16, kind=kind, n=n, c=c,
                                 block=block, block_q=block_q, block_k=block_k, shift=shift, fast_rho=fast_rho,
                                 inv_stat=inv_stat, compact_stat=compact_stat, poly_rho=poly_rho,
                                 range_guard=range_guard, resident_bwd=resident_bwd, diagonal_bwd=diagonal_bwd,
                                 head_resident=head_resident)
    if D != 64:
        raise ValueError(f"algx attention supports head_dim 64, got {D}")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (jnp.bfloat16, jnp.float32):
        raise ValueError("q, k, v must share one dtype, bfloat16 or float32")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must have the same (B, H, T, D) shape")
    has_sink = sink_logit is not None
    ints, floats = VA.config_lists(kind, var, T, D, c, has_sink, range_guard)
    if has_sink:
        s_in = jnp.asarray(sink_logit, jnp.float32)
        sink = jnp.broadcast_to(jnp.reshape(s_in, (-1,)), (H,)) / VA.sink_unit(kind, c)
    else:
        sink = jnp.zeros((0,), jnp.float32)
    return _flash(q, k, v, sink, tuple(ints), tuple(floats))
