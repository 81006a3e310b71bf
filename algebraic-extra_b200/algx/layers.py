"""Row RMS norm, SwiGLU and ALU-GLU over libalgx, as autograd functions.

These are the model's own elementwise layers around the three hot kernels
(model.py:158-159 ``_norm``; model.py:193-198 ``gate * silu(up)`` or
``gate * alu(up)``), each one fused launch forward and one backward, for the
config-5 training step in ``algx.model``. Like the hot kernels they run on
CUDA tensors only.
"""

from __future__ import annotations

import torch

from . import _lib as L


def rmsnorm_forward(x: torch.Tensor, gain, eps: float) -> torch.Tensor:
    """y = rms_norm(x) * gain over the last axis (algebraic.py:76-83), one launch."""
    dim = x.shape[-1]
    y = torch.empty_like(x)
    L.check(L.lib().algx_rmsnorm_fwd(x.data_ptr(), L.ptr(gain), y.data_ptr(), x.numel() // dim, dim,
                                     L.dtype_code(x.dtype), float(eps), L.stream_of(x)), "algx_rmsnorm_fwd")
    return y


def rmsnorm_backward(x: torch.Tensor, gain, dy: torch.Tensor, eps: float):
    """(dx, dgain) of ``rmsnorm_forward``; dgain is None without a gain."""
    dim = x.shape[-1]
    rows = x.numel() // dim
    dy = dy.to(x.dtype).contiguous()
    dx = torch.empty_like(x)
    lib = L.lib()
    dgain = None
    ws, nbytes = None, 0
    if gain is not None:
        dgain = torch.empty(dim, dtype=torch.float32, device=x.device)
        nbytes = lib.algx_rmsnorm_bwd_workspace_size(rows, dim)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    L.check(lib.algx_rmsnorm_bwd(x.data_ptr(), L.ptr(gain), dy.data_ptr(), dx.data_ptr(), L.ptr(dgain), rows, dim,
                                 L.dtype_code(x.dtype), float(eps), L.ptr(ws), nbytes, L.stream_of(x)),
            "algx_rmsnorm_bwd")
    return dx, dgain


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gain, eps):
        xc = x.contiguous()
        ctx.eps = float(eps)
        ctx.has_gain = gain is not None
        ctx.save_for_backward(xc, gain)
        return rmsnorm_forward(xc, gain, eps)

    @staticmethod
    def backward(ctx, dy):
        x, gain = ctx.saved_tensors
        dx, dgain = rmsnorm_backward(x, gain if ctx.has_gain else None, dy, ctx.eps)
        return dx, (dgain.to(gain.dtype) if dgain is not None else None), None


def rms_norm(x: torch.Tensor, gain, eps: float = 1e-5) -> torch.Tensor:
    """``algebraic.rms_norm`` (algebraic.py:76-83): fp32 maths, result in x's dtype.

    ``gain`` is a float32 vector of the last axis' length, or None for the
    parameter-free form. The width must be a multiple of 16 bytes and at most
    4096 (bf16) / 2048 (float32).
    """
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("rms_norm needs float32 or bfloat16 input")
    if gain is not None and (gain.dtype != torch.float32 or tuple(gain.shape) != (x.shape[-1],)):
        raise ValueError("rms_norm gain must be float32 with the width of x's last axis")
    if eps <= 0:
        raise ValueError("rms_norm epsilon must be positive")
    L.require_cuda(x, gain)
    return _RMSNorm.apply(x, gain, float(eps))


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        ff = gu.shape[-1] // 2
        rows = gu.numel() // gu.shape[-1]
        y = torch.empty(gu.shape[:-1] + (ff,), dtype=gu.dtype, device=gu.device)
        L.check(L.lib().algx_swiglu_fwd(gu.data_ptr(), y.data_ptr(), rows, ff, L.stream_of(gu)), "algx_swiglu_fwd")
        ctx.save_for_backward(gu)
        return y

    @staticmethod
    def backward(ctx, dy):
        (gu,) = ctx.saved_tensors
        ff = gu.shape[-1] // 2
        rows = gu.numel() // gu.shape[-1]
        dy = dy.to(gu.dtype).contiguous()
        dgu = torch.empty_like(gu)
        L.check(L.lib().algx_swiglu_bwd(gu.data_ptr(), dy.data_ptr(), dgu.data_ptr(), rows, ff, L.stream_of(gu)),
                "algx_swiglu_bwd")
        return dgu


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """``gate * silu(up)`` for ``gu = [gate | up]`` on the last axis (model.py:193-198), bf16.

    ``gu`` is the output of one GEMM against ``[w_g | w_u]``; the result has
    half its last axis.
    """
    if gu.dtype != torch.bfloat16:
        raise ValueError("swiglu needs bfloat16 input")
    if gu.shape[-1] % 16:
        raise ValueError("swiglu needs an even hidden width that is a multiple of 8")
    L.require_cuda(gu)
    return _SwiGLU.apply(gu)


class _ALUGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu, beta):
        gu = gu.contiguous()
        ff = gu.shape[-1] // 2
        rows = gu.numel() // gu.shape[-1]
        y = torch.empty(gu.shape[:-1] + (ff,), dtype=gu.dtype, device=gu.device)
        L.check(L.lib().algx_aluglu_fwd(gu.data_ptr(), y.data_ptr(), rows, ff, float(beta), L.stream_of(gu)),
                "algx_aluglu_fwd")
        ctx.save_for_backward(gu)
        ctx.beta = float(beta)
        return y

    @staticmethod
    def backward(ctx, dy):
        (gu,) = ctx.saved_tensors
        ff = gu.shape[-1] // 2
        rows = gu.numel() // gu.shape[-1]
        dy = dy.to(gu.dtype).contiguous()
        dgu = torch.empty_like(gu)
        L.check(L.lib().algx_aluglu_bwd(gu.data_ptr(), dy.data_ptr(), dgu.data_ptr(), rows, ff, ctx.beta,
                                        L.stream_of(gu)), "algx_aluglu_bwd")
        return dgu, None


def aluglu(gu: torch.Tensor, beta: float = 1.0) -> torch.Tensor:
    """``gate * alu(up, beta)`` for ``gu = [gate | up]`` on the last axis (model.py:196-197,
    algebraic.py:86-113), bf16: the algebraic preset's gate (``ffn="alu_glu"``)."""
    if gu.dtype != torch.bfloat16:
        raise ValueError("aluglu needs bfloat16 input")
    if gu.shape[-1] % 16:
        raise ValueError("aluglu needs an even hidden width that is a multiple of 8")
    L.require_cuda(gu)
    return _ALUGLU.apply(gu, float(beta))


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, w16):
        ctx.save_for_backward(x, w16)
        return x @ w16

    @staticmethod
    def backward(ctx, dy):
        x, w16 = ctx.saved_tensors
        dx = dy @ w16.t()
        x2 = x.reshape(-1, x.shape[-1])
        dy2 = dy.reshape(-1, dy.shape[-1])
        dw = torch.mm(x2.t(), dy2, out_dtype=torch.float32)
        return dx, dw, None


def linear(x: torch.Tensor, w: torch.Tensor, w16: torch.Tensor) -> torch.Tensor:
    """``x @ w.astype(bf16)`` (model.py:167-198) for a float32 master ``w`` whose
    bf16 copy ``w16`` the caller keeps for a whole optimizer step: the weight is
    not cast again per micro-batch, and the weight gradient comes out of its
    GEMM in float32 (no bf16 rounding of it, no separate cast kernel) to be
    accumulated into the master's gradient."""
    return _Linear.apply(x, w, w16)


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, gain, eps):
        x, r = x.contiguous(), r.contiguous()
        dim = x.shape[-1]
        s = torch.empty_like(x)
        y = torch.empty_like(x)
        L.check(L.lib().algx_add_rmsnorm_fwd(x.data_ptr(), r.data_ptr(), L.ptr(gain), s.data_ptr(), y.data_ptr(),
                                             x.numel() // dim, dim, L.dtype_code(x.dtype), float(eps),
                                             L.stream_of(x)), "algx_add_rmsnorm_fwd")
        ctx.eps = float(eps)
        ctx.has_gain = gain is not None
        ctx.save_for_backward(s, gain)
        return s, y

    @staticmethod
    def backward(ctx, ds, dy):
        s, gain = ctx.saved_tensors
        gain = gain if ctx.has_gain else None
        if dy is None:
            return ds, ds, None, None
        if ds is None:
            dx, dgain = rmsnorm_backward(s, gain, dy, ctx.eps)
        else:
            dim = s.shape[-1]
            rows = s.numel() // dim
            dy = dy.to(s.dtype).contiguous()
            ds = ds.to(s.dtype).contiguous()
            dx = torch.empty_like(s)
            lib = L.lib()
            dgain, ws, nbytes = None, None, 0
            if gain is not None:
                dgain = torch.empty(dim, dtype=torch.float32, device=s.device)
                nbytes = lib.algx_rmsnorm_bwd_workspace_size(rows, dim)
                ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=s.device)
            L.check(lib.algx_add_rmsnorm_bwd(s.data_ptr(), L.ptr(gain), dy.data_ptr(), ds.data_ptr(), dx.data_ptr(),
                                             L.ptr(dgain), rows, dim, L.dtype_code(s.dtype), ctx.eps, L.ptr(ws),
                                             nbytes, L.stream_of(s)), "algx_add_rmsnorm_bwd")
        return dx, dx, (dgain.to(gain.dtype) if dgain is not None else None), None


def add_rms_norm(x: torch.Tensor, r: torch.Tensor, gain, eps: float = 1e-5):
    """``s = x + r; (s, rms_norm(s, gain))`` in one launch each way (the residual
    add and the norm that reads it, model.py:180-200); same values as the
    composed ops, with the backward's two gradient contributions to ``s``
    summed before one rounding."""
    if x.shape != r.shape or x.dtype != r.dtype:
        raise ValueError("add_rms_norm needs x and r of one shape and dtype")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("add_rms_norm needs float32 or bfloat16 input")
    if gain is not None and (gain.dtype != torch.float32 or tuple(gain.shape) != (x.shape[-1],)):
        raise ValueError("add_rms_norm gain must be float32 with the width of x's last axis")
    L.require_cuda(x, r, gain)
    return _AddRMSNorm.apply(x, r, gain, float(eps))
