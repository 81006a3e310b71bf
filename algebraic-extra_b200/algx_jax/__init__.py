"""algx_jax: the algx kernels behind JAX, through XLA FFI custom calls.

Drop-in replacements for the reference's ``algebraic.kernels`` entry points,
with the same signatures and custom VJPs:

* ``algx_jax.flash.flash_attention``   (kernels/flash.py:763)
* ``algx_jax.fused_head.fused_head``   (kernels/fused_head.py:260)
* ``algx_jax.qk_norm.qk_rms_norm``     (kernels/qk_norm.py:62)

The handlers (jax_ffi/algx_jax_ffi.cc) are built into
``algx/libalgx_jax.so`` by ``jax_ffi/build.py`` where jaxlib is installed;
the targets are registered for the CUDA platform on first use. There is no
CPU fallback.
"""

from .flash import flash_attention  # noqa: F401
from .fused_head import fused_head  # noqa: F401
from .qk_norm import qk_rms_norm  # noqa: F401
