"""``torch.library`` operators over libalgx (the framework-level front-end).

The three hot-path families are registered as custom operators in the
``algx`` namespace, each with a fake (shape-only) implementation and its
backward wired through ``torch.library.register_autograd``:

* ``algx::qk_rms_norm`` / ``algx::qk_rms_norm_backward``
* ``algx::flash_attention_fwd`` / ``algx::flash_attention_bwd``
* ``algx::fused_head_fwd`` / ``algx::fused_head_bwd``

To a tracer (``torch.compile``, ``torch.export``, CUDA-graph capture tools)
each call is one opaque node with known output shapes, where the
``autograd.Function`` wrappers of ``algx.kernels`` would be traced through.
The public functions below take the same arguments, raise the same errors
and return the same values as ``algx.kernels.{qk_norm,flash,fused_head}``,
which mirror the reference's kernels/qk_norm.py:62, kernels/flash.py:763 and
kernels/fused_head.py:260.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import Tensor

from . import _lib as L
from .kernels import flash as F
from .kernels import fused_head as FH
from .kernels import qk_norm as Q


# ------------------------------------------------------------------ QK norm
@torch.library.custom_op("algx::qk_rms_norm", mutates_args=())
def _qk_rms_norm_op(x: Tensor, gain: Tensor, eps: float) -> Tensor:
    return Q.qknorm_forward(x.contiguous(), gain, eps)


@_qk_rms_norm_op.register_fake
def _(x, gain, eps):
    return torch.empty_like(x)


@torch.library.custom_op("algx::qk_rms_norm_backward", mutates_args=())
def _qk_rms_norm_bwd_op(x: Tensor, gain: Tensor, dy: Tensor, eps: float) -> Tuple[Tensor, Tensor]:
    return Q.qknorm_backward(x.contiguous(), gain, dy, eps)


@_qk_rms_norm_bwd_op.register_fake
def _(x, gain, dy, eps):
    return torch.empty_like(x), gain.new_empty((64,), dtype=torch.float32)


def _qk_setup(ctx, inputs, output):
    x, gain, eps = inputs
    ctx.save_for_backward(x, gain)
    ctx.eps = eps


def _qk_backward(ctx, dy):
    x, gain = ctx.saved_tensors
    dx, dgain = _qk_rms_norm_bwd_op(x, gain, dy, ctx.eps)
    return dx, dgain.to(gain.dtype), None


torch.library.register_autograd("algx::qk_rms_norm", _qk_backward, setup_context=_qk_setup)


def qk_rms_norm(x, gain, eps=1e-5, *, block=1024):
    """``algx.kernels.qk_norm.qk_rms_norm`` as one ``algx::qk_rms_norm`` node."""
    if x.ndim < 2 or x.shape[-1] != 64 or tuple(gain.shape) != (64,):
        raise ValueError("QK RMS kernel needs D=64 and a one-dimensional gain")
    if x.dtype not in (torch.bfloat16, torch.float32) or gain.dtype != torch.float32:
        raise ValueError("QK RMS kernel needs float32/BF16 input and float32 gain")
    if block < 8 or block % 8 or (x.numel() // 64) % block:
        raise ValueError("QK RMS row count must be divisible by a block aligned to eight rows")
    if eps <= 0:
        raise ValueError("QK RMS epsilon must be positive")
    L.require_cuda(x, gain)
    return _qk_rms_norm_op(x, gain.contiguous(), float(eps))


# ------------------------------------------------------------------ attention
# The resolved variant travels as plain scalars (a custom operator's schema
# has no place for the ctypes struct): kind, mode, n, fast_rho, inv_stat,
# has_sink as ints; clamp, scale and the three guard bounds as floats.
# The ctypes struct is built only inside the operators, so a tracer sees no
# ctypes object; the lists come from the same resolution as the eager path.
_cfg = F.config_from_lists


@torch.compiler.assume_constant_result
def _attn_lists(kind, n, c, T, D, shift, fast_rho, inv_stat, compact_stat, poly_rho, range_guard, has_sink):
    var = F.make_variant(kind, n, c, T, shift, fast_rho, inv_stat, compact_stat, poly_rho)
    if range_guard and kind == "asinh" and n <= 32 and poly_rho:
        raise ValueError("range_guard is for exact radical evaluation")
    return F.config_lists(kind, var, T, D, c, has_sink, range_guard)


def _guarded(ints: List[int]) -> bool:
    return ints[0] == L.ALGX_ATTN_ASINH and ints[1] == L.ALGX_MODE_GUARDED


@torch.library.custom_op("algx::flash_attention_fwd", mutates_args=())
def _attn_fwd_op(q: Tensor, k: Tensor, v: Tensor, sink: Optional[Tensor], ints: List[int],
                 floats: List[float]) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    o, saved = F.attn_forward(q, k, v, sink, _cfg(ints, floats))
    q_s, _, _, _, _, o_prec, stat, guard = saved
    if o_prec is None:
        o_prec = q.new_empty((0,), dtype=torch.float32)
    return o, q_s, stat, guard, o_prec


@_attn_fwd_op.register_fake
def _(q, k, v, sink, ints, floats):
    B, H, T, D = q.shape
    prec_shape = (B, H, T, D) if _guarded(ints) else (0,)
    return (torch.empty_like(q), torch.empty_like(q), q.new_empty((B, H, T), dtype=torch.float32),
            q.new_empty((4,), dtype=torch.float32), q.new_empty(prec_shape, dtype=torch.float32))


@torch.library.custom_op("algx::flash_attention_bwd", mutates_args=())
def _attn_bwd_op(q_s: Tensor, k: Tensor, v: Tensor, sink: Optional[Tensor], o: Tensor, o_prec: Tensor,
                 stat: Tensor, guard: Tensor, do: Tensor, ints: List[int],
                 floats: List[float]) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    saved = (q_s, k, v, sink, o, o_prec if o_prec.numel() else None, stat, guard)
    dq, dk, dv, dsink = F.attn_backward(saved, _cfg(ints, floats), do)
    if dsink is None:
        dsink = q_s.new_empty((0,), dtype=torch.float32)
    return dq, dk, dv, dsink


@_attn_bwd_op.register_fake
def _(q_s, k, v, sink, o, o_prec, stat, guard, do, ints, floats):
    H = q_s.shape[1]
    dsink_shape = (H,) if sink is not None else (0,)
    return (torch.empty_like(q_s), torch.empty_like(k), torch.empty_like(v),
            q_s.new_empty(dsink_shape, dtype=torch.float32))


def _attn_setup(ctx, inputs, output):
    q, k, v, sink, ints, floats = inputs
    o, q_s, stat, guard, o_prec = output
    ctx.save_for_backward(q_s, k, v, sink, o, o_prec, stat, guard)
    ctx.ints, ctx.floats = ints, floats
    ctx.has_sink = sink is not None


def _attn_backward(ctx, do, _dq_s, _dstat, _dguard, _dprec):
    q_s, k, v, sink, o, o_prec, stat, guard = ctx.saved_tensors
    dq, dk, dv, dsink = _attn_bwd_op(q_s, k, v, sink, o, o_prec, stat, guard, do.contiguous(), ctx.ints,
                                     ctx.floats)
    return dq, dk, dv, (dsink if ctx.has_sink else None), None, None


torch.library.register_autograd("algx::flash_attention_fwd", _attn_backward, setup_context=_attn_setup)


def flash_attention(q, k, v, sink_logit=None, *, kind: str = "softmax", n: int = 16, c: float = 16.0,
                    block: int = 512, block_q: Optional[int] = None, block_k: Optional[int] = None,
                    shift: Optional[bool] = None, fast_rho: Optional[bool] = None,
                    inv_stat: Optional[bool] = None, compact_stat: bool = True, poly_rho: bool = False,
                    range_guard: bool = False, resident_bwd: Optional[bool] = None,
                    diagonal_bwd: Optional[bool] = None, diagonal_fwd: Optional[bool] = None,
                    head_resident: Optional[bool] = None):
    """``algx.kernels.flash.flash_attention`` as one ``algx::flash_attention_fwd`` node."""
    B, H, T, D = q.shape
    bq = min(block_q or block, T)
    bk = min(block_k or block, T)
    if T % bq or T % bk:
        raise ValueError(f"sequence length {T} must be divisible by blocks ({bq}, {bk})")
    sink = F.check_inputs(q, k, v, sink_logit, kind, c)
    ints, floats = _attn_lists(kind, n, c, T, D, shift, fast_rho, inv_stat, compact_stat, poly_rho, range_guard,
                               sink is not None)
    o, *_ = _attn_fwd_op(q.contiguous(), k.contiguous(), v.contiguous(), sink, ints, floats)
    return o


# ------------------------------------------------------------------ fused head
# ints [kind, n, has_ignore, ignore_index]; floats [inv_c, clamp, slope], slope
# being d(objective)/d(mean per-token term): 1 for ce, n / c for alg_ce.
_head_cfg = FH.head_config_from_lists


@torch.compiler.assume_constant_result
def _head_lists(kind, n, c, vocab, ignore_index):
    ints, floats = FH.head_config_lists(kind, n, c, vocab, ignore_index)
    return ints, floats + [1.0 if kind == "ce" else n / c]


# h and embed enter in their own dtypes and are rounded to bfloat16 inside the
# operators (as kernels/fused_head.py:103 does), so dh and dE come back in those
# dtypes.
def _bf16(h: Tensor, embed: Tensor, targets: Tensor):
    return (h.to(torch.bfloat16).contiguous(), embed.to(torch.bfloat16).contiguous(),
            targets.to(torch.int32).contiguous())


@torch.library.custom_op("algx::fused_head_fwd", mutates_args=())
def _head_fwd_op(h: Tensor, embed: Tensor, targets: Tensor, ints: List[int],
                 floats: List[float]) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    cfg = _head_cfg(ints, floats)
    h16, e16, t32 = _bf16(h, embed, targets)
    mlz = FH.head_forward_partials(h16, e16, t32, cfg)
    stat, tel, obj, count = FH.head_finalize(cfg, t32, mlz, e16.shape[0])
    return obj.reshape(()), tel, stat, count


@_head_fwd_op.register_fake
def _(h, embed, targets, ints, floats):
    N = h.shape[0]
    f32 = torch.float32
    return (h.new_empty((), dtype=f32), h.new_empty((N,), dtype=f32), h.new_empty((N,), dtype=f32),
            h.new_empty((1,), dtype=f32))


@torch.library.custom_op("algx::fused_head_bwd", mutates_args=())
def _head_bwd_op(h: Tensor, embed: Tensor, targets: Tensor, stat: Tensor, scale: Tensor, ints: List[int],
                 floats: List[float]) -> Tuple[Tensor, Tensor]:
    h16, e16, t32 = _bf16(h, embed, targets)
    dh, de = FH.head_backward(h16, e16, t32, stat, scale, _head_cfg(ints, floats))
    return dh.to(h.dtype), de.to(embed.dtype)


@_head_bwd_op.register_fake
def _(h, embed, targets, stat, scale, ints, floats):
    return torch.empty_like(h), torch.empty_like(embed)


def _head_setup(ctx, inputs, output):
    h, embed, targets, ints, floats = inputs
    obj, tel, stat, count = output
    ctx.save_for_backward(h, embed, targets, stat, count)
    ctx.ints, ctx.floats = ints, floats


def _head_backward(ctx, g_obj, _g_tel, _g_stat, _g_count):
    h, embed, targets, stat, count = ctx.saved_tensors
    scale = (g_obj.reshape(1).float() * ctx.floats[2] / count).contiguous()
    dh, de = _head_bwd_op(h, embed, targets, stat, scale, ctx.ints, ctx.floats)
    return dh, de, None, None, None


torch.library.register_autograd("algx::fused_head_fwd", _head_backward, setup_context=_head_setup)


def fused_head(h, embed, targets, *, kind="ce", n=16, c=16.0, block_n=128, block_v=512, ignore_index=None):
    """``algx.kernels.fused_head.fused_head`` as one ``algx::fused_head_fwd`` node."""
    if kind not in ("ce", "alg_ce"):
        raise ValueError(kind)
    if kind == "alg_ce" and (n & (n - 1)):
        raise ValueError("n must be a power of two")
    N, d = h.shape
    bn = min(block_n, N)
    if N % bn:
        raise ValueError(f"token count {N} must be divisible by block {bn}")
    if kind == "alg_ce" and n not in (2, 4, 8, 16, 32):
        raise ValueError("algx fused head supports alg_ce powers n in {2, 4, 8, 16, 32}")
    if d % 64:
        raise ValueError(f"algx fused head needs d to be a multiple of 64, got {d}")
    if embed.shape[1] != d or targets.shape != (N,):
        raise ValueError("h (N, d), embed (V, d) and targets (N,) shapes disagree")
    L.require_cuda(h, embed, targets)
    ints, floats = _head_lists(kind, n, c, embed.shape[0], ignore_index)
    obj, tel, _, _ = _head_fwd_op(h, embed, targets, ints, floats)
    return obj, tel.detach()
