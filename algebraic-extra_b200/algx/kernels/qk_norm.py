"""QK RMS normalisation (drop-in for kernels/qk_norm.py:62-76).

Forward ``y = rms_norm(x) * gain`` and its VJP (dx by the AD formula of
algebraic.py:76-83, dgain = sum over rows of dy * x * tau) run in libalgx.
"""

import torch

from .. import _lib as L


def qknorm_forward(x, gain, eps):
    """y = rms_norm(x) * gain (one launch)."""
    y = torch.empty_like(x)
    L.check(L.lib().algx_qknorm_fwd(x.data_ptr(), gain.data_ptr(), y.data_ptr(), x.numel() // 64, 64,
                                    L.dtype_code(x.dtype), float(eps), L.stream_of(x)), "algx_qknorm_fwd")
    return y


def qknorm_backward(x, gain, dy, eps, workspace=None):
    """(dx, dgain) of the QK norm (two launches: rows, then the fixed-order dgain sum)."""
    dy = dy.to(x.dtype).contiguous()
    rows = x.numel() // 64
    dx = torch.empty_like(x)
    dgain = torch.empty(64, dtype=torch.float32, device=x.device)
    nbytes = L.lib().algx_qknorm_bwd_workspace_size(rows, 64)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    L.check(L.lib().algx_qknorm_bwd(x.data_ptr(), gain.data_ptr(), dy.data_ptr(), dx.data_ptr(),
                                    dgain.data_ptr(), rows, 64, L.dtype_code(x.dtype), float(eps),
                                    workspace.data_ptr(), nbytes, L.stream_of(x)), "algx_qknorm_bwd")
    return dx, dgain


class _QKNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gain, eps):
        xc = x.contiguous()
        y = qknorm_forward(xc, gain, eps)
        ctx.save_for_backward(xc, gain)
        ctx.eps = float(eps)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gain = ctx.saved_tensors
        dx, dgain = qknorm_backward(x, gain, dy, ctx.eps)
        return dx, dgain.to(gain.dtype), None


def qk_rms_norm(x, gain, eps=1e-5, *, block=1024):
    """RMS-normalize D=64 rows with a learned gain (kernels/qk_norm.py:62-76).

    ``block`` is validated as the reference does (rows divisible by a block
    aligned to eight rows) but does not change the result: the CUDA kernel
    picks its own tiling.
    """
    if x.ndim < 2 or x.shape[-1] != 64 or tuple(gain.shape) != (64,):
        raise ValueError("QK RMS kernel needs D=64 and a one-dimensional gain")
    if x.dtype not in (torch.bfloat16, torch.float32) or gain.dtype != torch.float32:
        raise ValueError("QK RMS kernel needs float32/BF16 input and float32 gain")
    if block < 8 or block % 8 or (x.numel() // 64) % block:
        raise ValueError("QK RMS row count must be divisible by a block aligned to eight rows")
    if eps <= 0:
        raise ValueError("QK RMS epsilon must be positive")
    L.require_cuda(x, gain)
    return _QKNorm.apply(x, gain.contiguous(), float(eps))
