"""``qk_rms_norm`` for JAX over libalgx (drop-in for kernels/qk_norm.py:62-76).

Same signature, checks and ``custom_vjp`` structure as the reference; the
Pallas calls are replaced by the XLA FFI targets ``algx_qknorm_fwd`` and
``algx_qknorm_bwd`` (jax_ffi/algx_jax_ffi.cc).
"""

from __future__ import annotations

import functools

import jax
import jax.numpy as jnp
import numpy as np

from algx import variants as VA

from . import _ffi


def _norm_fwd_call(x, gain, eps):
    _ffi.libs()
    return jax.ffi.ffi_call("algx_qknorm_fwd", jax.ShapeDtypeStruct(x.shape, x.dtype))(x, gain, eps=np.float32(eps))


@functools.partial(jax.custom_vjp, nondiff_argnums=(2,))
def _qk_norm(x, gain, eps):
    return _norm_fwd_call(x, gain, eps)


def _qk_norm_fwd(x, gain, eps):
    return _norm_fwd_call(x, gain, eps), (x, gain)


def _qk_norm_bwd(eps, res, dy):
    x, gain = res
    rows = x.size // 64
    ws = max(int(_ffi.core().algx_qknorm_bwd_workspace_size(rows, 64)), 1)
    dx, dgain, _ = jax.ffi.ffi_call(
        "algx_qknorm_bwd",
        (jax.ShapeDtypeStruct(x.shape, x.dtype), jax.ShapeDtypeStruct((64,), jnp.float32),
         jax.ShapeDtypeStruct((ws,), jnp.uint8)))(x, gain, dy.astype(x.dtype), eps=np.float32(eps))
    return dx, dgain.astype(gain.dtype)


_qk_norm.defvjp(_qk_norm_fwd, _qk_norm_bwd)


def qk_rms_norm(x, gain, eps=1e-5, *, block=1024):
    """RMS-normalize D=64 rows with a learned gain (kernels/qk_norm.py:62-76)."""
    x = jnp.asarray(x)
    gain = jnp.asarray(gain)
    VA.check_qk_norm_options(x.shape, x.shape[-1] if x.ndim else 0, gain.shape,
                             x.dtype in (jnp.bfloat16, jnp.float32), gain.dtype == jnp.float32, block, eps)
    return _qk_norm(x, gain, float(eps))
