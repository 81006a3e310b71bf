"""algx: B200-native (sm_100a) kernels for the Algebraic Transformer hot path.

Public API, mirroring the reference's ``algebraic.kernels`` modules:

* ``algx.kernels.flash.flash_attention``    (kernels/flash.py:763)
* ``algx.kernels.fused_head.fused_head``    (kernels/fused_head.py:260)
* ``algx.kernels.qk_norm.qk_rms_norm``      (kernels/qk_norm.py:62)

All three are torch ``autograd.Function``s over the C ABI of ``libalgx.so``.
``algx.torch_ops`` registers the same three families as ``torch.library``
operators (``torch.ops.algx.*``) for tracers that need opaque nodes.
"""

__version__ = "0.1.0"
