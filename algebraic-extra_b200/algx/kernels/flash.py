"""Causal flash attention, softmax and asinh-power kinds (drop-in for kernels/flash.py).

Same call signature, variant resolution and ValueError conditions as the
reference's ``flash_attention`` (kernels/flash.py:732-857). The schedule
knobs of the TPU kernels (``block*``, ``resident_bwd``, ``diagonal_*``,
``head_resident``, ``compact_stat``) are validated exactly as the reference
validates them and otherwise ignored: the sm_100a kernels choose their own
tiles, and none of those knobs changes the function computed.

The range guard (``range_guard=True``) is evaluated on the device:
``algx_attn_prepare`` folds the score scale into q and writes the guard
maxima, and the forward/backward kernels pick the unshifted (low) or the
shifted (high) branch from them, so no host synchronisation happens.
"""

from __future__ import annotations

import math  # noqa: F401
from typing import Optional

import torch

from .. import _lib as L


# Variant resolution, option checks and wrapper constants live in the
# torch-free algx.variants (shared with the JAX front-end); re-exported here.
from ..variants import Variant, check_flash_options, config_lists, make_variant  # noqa: E402,F401


def attn_forward(q, k, v, sink, cfg: L.AttnConfig):
    """Forward launch group (prepare + forward); returns (o, saved residuals)."""
    B, H, T, D = q.shape
    q_s = torch.empty_like(q)
    guard = torch.empty(4, dtype=torch.float32, device=q.device)
    sp = sink.data_ptr() if sink is not None else None
    L.check(L.lib().algx_attn_prepare(cfg, q.data_ptr(), k.data_ptr(), v.data_ptr(), sp, q_s.data_ptr(),
                                      guard.data_ptr(), B, H, T, D, L.dtype_code(q.dtype), L.stream_of(q)),
            "algx_attn_prepare")
    return attn_forward_prepared(q_s, k, v, sink, guard, cfg)


def _rot_args(rotary):
    if rotary is None:
        return None, None, 0
    cos, sin = rotary
    return cos.data_ptr(), sin.data_ptr(), cos.shape[0]


def qknorm_attn_prepare(q, k, v, gain_q, gain_k, sink, cfg: L.AttnConfig, eps: float, rotary=None):
    """The fused QK-norm (-> rotary) prologue alone: (q_scaled, k_norm, guard maxima).
    ``rotary``: None or (cos, sin), contiguous fp32 (>= T, 32) on q's device."""
    B, H, T, D = q.shape
    q_s = torch.empty_like(q)
    k_n = torch.empty_like(k)
    guard = torch.empty(4, dtype=torch.float32, device=q.device)
    sp = sink.data_ptr() if sink is not None else None
    L.check(L.lib().algx_qknorm_attn_prepare(cfg, q.data_ptr(), k.data_ptr(), v.data_ptr(), gain_q.data_ptr(),
                                             gain_k.data_ptr(), *_rot_args(rotary), sp, q_s.data_ptr(),
                                             k_n.data_ptr(), guard.data_ptr(), B, H, T, D, L.dtype_code(q.dtype),
                                             float(eps), L.stream_of(q)), "algx_qknorm_attn_prepare")
    return q_s, k_n, guard


def attn_forward_qknorm(q, k, v, gain_q, gain_k, sink, cfg: L.AttnConfig, eps: float, rotary=None):
    """Forward launch group with the fused QK-norm prologue: attention of
    (rms_norm(q) * gain_q, rms_norm(k) * gain_k, v), rotated by ``rotary``
    when given, with the QK norm, the rotation, the scale fold and the guard
    maxima in one launch; returns (o, saved)."""
    q_s, k_n, guard = qknorm_attn_prepare(q, k, v, gain_q, gain_k, sink, cfg, eps, rotary)
    return attn_forward_prepared(q_s, k_n, v, sink, guard, cfg)


def attn_forward_prepared(q_s, k, v, sink, guard, cfg: L.AttnConfig):
    """Forward kernels on prepared inputs (q_scaled, the guard maxima); (o, saved)."""
    B, H, T, D = q_s.shape
    q = q_s
    dt = L.dtype_code(q.dtype)
    st = L.stream_of(q)
    sp = sink.data_ptr() if sink is not None else None
    o = torch.empty_like(q)
    stat = torch.empty((B, H, T), dtype=torch.float32, device=q.device)
    o_prec = None
    if cfg.kind == L.ALGX_ATTN_ASINH and cfg.mode == L.ALGX_MODE_GUARDED:
        o_prec = torch.empty((B, H, T, D), dtype=torch.float32, device=q.device)
    L.check(L.lib().algx_attn_fwd(cfg, q_s.data_ptr(), k.data_ptr(), v.data_ptr(), sp, guard.data_ptr(),
                                  o.data_ptr(), L.ptr(o_prec), stat.data_ptr(), B, H, T, D, dt, st),
            "algx_attn_fwd")
    return o, (q_s, k, v, sink, o, o_prec, stat, guard)


def attn_backward(saved, cfg: L.AttnConfig, do, workspace=None):
    """Backward launch group; returns (dq, dk, dv, dsink)."""
    q_s, k, v, sink, o, o_prec, stat, guard = saved
    B, H, T, D = q_s.shape
    do = do.to(q_s.dtype).contiguous()
    dq = torch.empty_like(q_s)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    dsink = torch.empty(H, dtype=torch.float32, device=q_s.device) if sink is not None else None
    nbytes = L.lib().algx_attn_bwd_workspace_size(B, H, T, D)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q_s.device)
    L.check(L.lib().algx_attn_bwd(cfg, q_s.data_ptr(), k.data_ptr(), v.data_ptr(), L.ptr(sink),
                                  guard.data_ptr(), o.data_ptr(), L.ptr(o_prec), stat.data_ptr(),
                                  do.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), L.ptr(dsink),
                                  B, H, T, D, L.dtype_code(q_s.dtype), workspace.data_ptr(), nbytes,
                                  L.stream_of(q_s)), "algx_attn_bwd")
    return dq, dk, dv, dsink


def qknorm_attn_backward(q, k, gain_q, gain_k, saved, cfg: L.AttnConfig, do, eps: float, workspace=None,
                         rotary=None):
    """Backward launch group of :func:`attn_forward_qknorm`: the attention
    backward and the QK-norm backward of q and k with the latter fused into
    one epilogue launch; returns (dq, dk, dv, dgain_q, dgain_k, dsink) with
    dq, dk the gradients of the raw (pre-norm) q, k."""
    q_s, k_n, v, sink, o, o_prec, stat, guard = saved
    B, H, T, D = q_s.shape
    do = do.to(q_s.dtype).contiguous()
    dq = torch.empty_like(q_s)
    dk = torch.empty_like(k_n)
    dv = torch.empty_like(v)
    dgq = torch.empty(D, dtype=torch.float32, device=q_s.device)
    dgk = torch.empty(D, dtype=torch.float32, device=q_s.device)
    dsink = torch.empty(H, dtype=torch.float32, device=q_s.device) if sink is not None else None
    nbytes = L.lib().algx_qknorm_attn_bwd_workspace_size(B, H, T, D)
    if workspace is None or workspace.numel() < nbytes:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=q_s.device)
    L.check(L.lib().algx_qknorm_attn_bwd(cfg, q.data_ptr(), k.data_ptr(), gain_q.data_ptr(), gain_k.data_ptr(),
                                         *_rot_args(rotary), q_s.data_ptr(), k_n.data_ptr(), v.data_ptr(), L.ptr(sink), guard.data_ptr(),
                                         o.data_ptr(), L.ptr(o_prec), stat.data_ptr(), do.data_ptr(), dq.data_ptr(),
                                         dk.data_ptr(), dv.data_ptr(), dgq.data_ptr(), dgk.data_ptr(), L.ptr(dsink),
                                         B, H, T, D, L.dtype_code(q_s.dtype), float(eps), workspace.data_ptr(),
                                         nbytes, L.stream_of(q_s)), "algx_qknorm_attn_bwd")
    return dq, dk, dv, dgq, dgk, dsink


class _Flash(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, sink, cfg: L.AttnConfig):
        o, saved = attn_forward(q, k, v, sink, cfg)
        ctx.cfg = cfg
        ctx.save_for_backward(*saved)
        return o

    @staticmethod
    def backward(ctx, do):
        dq, dk, dv, dsink = attn_backward(ctx.saved_tensors, ctx.cfg, do)
        return dq, dk, dv, dsink, None


def config_from_lists(ints, floats) -> L.AttnConfig:
    """Pack :func:`config_lists` into the C ABI's ``AlgxAttnConfig``."""
    cfg = L.AttnConfig()
    cfg.kind, cfg.mode, cfg.n, cfg.fast_rho, cfg.inv_stat, cfg.has_sink = (int(i) for i in ints)
    cfg.clamp, cfg.scale, cfg.guard_qk, cfg.guard_sink, cfg.guard_v = (float(f) for f in floats)
    return cfg


def build_config(kind, var: Variant, T: int, D: int, c: float, has_sink: bool,
                 range_guard: bool) -> L.AttnConfig:
    """Pack the resolved variant and the wrapper constants (kernels/flash.py:823-856)."""
    return config_from_lists(*config_lists(kind, var, T, D, c, has_sink, range_guard))


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
    """Causal attention on (B, H, T, D); ``sink_logit`` broadcastable to (H,).

    Same semantics as the reference (kernels/flash.py:763-857). ``poly_rho``
    selects a TPU-only polynomial radical there; here it is validated the
    same way and the exact radical is evaluated (the same function, within
    the reference's own polynomial-mode tolerance). D must be 64.
    """
    B, H, T, D = q.shape
    var = check_flash_options(T, D, q.dtype == k.dtype == v.dtype == torch.bfloat16, kind=kind, n=n, c=c,
                              block=block, block_q=block_q, block_k=block_k, shift=shift, fast_rho=fast_rho,
                              inv_stat=inv_stat, compact_stat=compact_stat, poly_rho=poly_rho,
                              range_guard=range_guard, resident_bwd=resident_bwd, diagonal_bwd=diagonal_bwd,
                              head_resident=head_resident)
    cfg, sink = _checked_call(q, k, v, sink_logit, kind, var, c, range_guard)
    return _Flash.apply(q.contiguous(), k.contiguous(), v.contiguous(), sink, cfg)


def check_inputs(q, k, v, sink_logit, kind, c):
    """Shape / dtype / device checks shared by the public entry points; returns
    the sink logits divided by the score unit, broadcast to (H,), or None."""
    B, H, T, D = q.shape
    if D != 64:
        raise ValueError(f"algx attention supports head_dim 64, got {D}")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("q, k, v must share one dtype, bfloat16 or float32")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must have the same (B, H, T, D) shape")
    L.require_cuda(q, k, v)
    if sink_logit is None:
        return None
    unit = 1.0 if kind == "softmax" else float(c)
    s_in = torch.as_tensor(sink_logit, dtype=torch.float32, device=q.device)
    return (torch.broadcast_to(torch.reshape(s_in, (-1,)), (H,)) / unit).contiguous()


def _checked_call(q, k, v, sink_logit, kind, var, c, range_guard):
    """:func:`check_inputs` plus the packed configuration; (cfg, sink)."""
    sink = check_inputs(q, k, v, sink_logit, kind, c)
    B, H, T, D = q.shape
    return build_config(kind, var, T, D, c, sink is not None, range_guard), sink


class _QKNormFlash(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, gain_q, gain_k, sink, cfg: L.AttnConfig, eps: float, rotary):
        o, saved = attn_forward_qknorm(q, k, v, gain_q, gain_k, sink, cfg, eps, rotary)
        ctx.cfg, ctx.eps, ctx.rotary = cfg, eps, rotary
        ctx.save_for_backward(q, k, gain_q, gain_k, *saved)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, gain_q, gain_k, *saved = ctx.saved_tensors
        dxq, dxk, dv, dgq, dgk, dsink = qknorm_attn_backward(q, k, gain_q, gain_k, saved, ctx.cfg, do, ctx.eps,
                                                             rotary=ctx.rotary)
        return dxq, dxk, dv, dgq, dgk, dsink, None, None, None


def qknorm_flash_attention(q, k, v, gain_q, gain_k, sink_logit=None, *, eps: float = 1e-5,
                           kind: str = "asinh", n: int = 16, c: float = 16.0, block: int = 512,
                           range_guard: bool = False, shift: Optional[bool] = None,
                           fast_rho: Optional[bool] = None, inv_stat: Optional[bool] = None, rotary=None):
    """``flash_attention(rot(qk_rms_norm(q, gain_q, eps)), rot(qk_rms_norm(k, gain_k, eps)), v, sink_logit, ...)``
    with the QK norm, the rotation, the scale fold and the range-guard maxima
    fused into one prologue launch (model.py:170-174), and the QK-norm (and
    rotation) backward fused into one epilogue launch after the attention
    backward. ``rotary``: None (no rotation) or the (cos, sin) tables of
    ``apply_rotary`` (algebraic.py:172-179), each (>= T, 32); they are constants
    (no gradient). Same values and gradients (q, k, v, both gains and the sink)
    as the calls composed; the reference has no fused entry of this kind.
    """
    cfg, sink, gq, gk = qknorm_call_args(q, k, v, gain_q, gain_k, sink_logit, eps, kind, n, c, block, range_guard,
                                         shift, fast_rho, inv_stat)
    rot = rotary_tables(rotary, q)
    return _QKNormFlash.apply(q.contiguous(), k.contiguous(), v.contiguous(), gq, gk, sink, cfg, float(eps), rot)


def rotary_tables(rotary, q):
    """Validate (cos, sin) rotary tables for q (B, H, T, 64): fp32, contiguous, on q's device."""
    if rotary is None:
        return None
    cos, sin = rotary
    T, D = q.shape[-2], q.shape[-1]
    cos = torch.as_tensor(cos).to(device=q.device, dtype=torch.float32).contiguous()
    sin = torch.as_tensor(sin).to(device=q.device, dtype=torch.float32).contiguous()
    if cos.ndim != 2 or cos.shape != sin.shape or cos.shape[1] != D // 2 or cos.shape[0] < T:
        raise ValueError(f"rotary tables must both have shape (>= {T}, {D // 2}), got {tuple(cos.shape)} and "
                         f"{tuple(sin.shape)}")
    return cos, sin


def qknorm_call_args(q, k, v, gain_q, gain_k, sink_logit, eps, kind, n, c, block, range_guard, shift, fast_rho,
                     inv_stat):
    """Validation and configuration shared by the QK-norm attention entries: (cfg, sink, gain_q, gain_k)."""
    B, H, T, D = q.shape
    bq = min(block, T)
    if T % bq:
        raise ValueError(f"sequence length {T} must be divisible by blocks ({bq}, {bq})")
    if eps <= 0:
        raise ValueError("eps must be positive")
    var = make_variant(kind, n, c, T, shift, fast_rho, inv_stat, True, False)
    cfg, sink = _checked_call(q, k, v, sink_logit, kind, var, c, range_guard)
    gq = gain_q.to(device=q.device, dtype=torch.float32).contiguous()
    gk = gain_k.to(device=q.device, dtype=torch.float32).contiguous()
    if gq.shape != (64,) or gk.shape != (64,):
        raise ValueError("gains must have shape (64,)")
    return cfg, sink, gq, gk


# ------------------------------------------------------------ packed layout
def qknorm_attn_forward_packed(qkv, gain_q, gain_k, sink, cfg: L.AttnConfig, eps: float, rotary=None):
    """Forward launch group on the packed token-major qkv (B, T, 3, H, D):
    the prologue reads q, k, v in place and writes head-major q_scaled, k_norm
    and v; the attention kernels run head-major; the output is permuted to
    token-major (B, T, H, D). Returns (o_tokens, saved)."""
    B, T, _, H, D = qkv.shape
    lib = L.lib()
    dt = L.dtype_code(qkv.dtype)
    st = L.stream_of(qkv)
    q_s = torch.empty((B, H, T, D), dtype=qkv.dtype, device=qkv.device)
    k_n = torch.empty_like(q_s)
    v_h = torch.empty_like(q_s)
    guard = torch.empty(4, dtype=torch.float32, device=qkv.device)
    L.check(lib.algx_qknorm_attn_prepare_packed(cfg, qkv.data_ptr(), gain_q.data_ptr(), gain_k.data_ptr(),
                                                *_rot_args(rotary), L.ptr(sink), q_s.data_ptr(), k_n.data_ptr(),
                                                v_h.data_ptr(), guard.data_ptr(), B, H, T, D, dt, float(eps), st),
            "algx_qknorm_attn_prepare_packed")
    o, saved = attn_forward_prepared(q_s, k_n, v_h, sink, guard, cfg)
    o_tok = torch.empty((B, T, H, D), dtype=qkv.dtype, device=qkv.device)
    L.check(lib.algx_heads_to_tokens(o.data_ptr(), o_tok.data_ptr(), B, H, T, D, dt, st), "algx_heads_to_tokens")
    return o_tok, saved


def qknorm_attn_backward_packed(qkv, gain_q, gain_k, saved, cfg: L.AttnConfig, do_tok, eps: float, rotary=None):
    """Backward of :func:`qknorm_attn_forward_packed`: (dqkv, dgain_q, dgain_k, dsink)."""
    q_s, k_n, v_h, sink, o, o_prec, stat, guard = saved
    B, H, T, D = q_s.shape
    lib = L.lib()
    dt = L.dtype_code(q_s.dtype)
    st = L.stream_of(q_s)
    do_tok = do_tok.to(q_s.dtype).contiguous()
    do = torch.empty_like(q_s)
    L.check(lib.algx_tokens_to_heads(do_tok.data_ptr(), do.data_ptr(), B, H, T, D, dt, st), "algx_tokens_to_heads")
    dqkv = torch.empty_like(qkv)
    dgq = torch.empty(D, dtype=torch.float32, device=q_s.device)
    dgk = torch.empty(D, dtype=torch.float32, device=q_s.device)
    dsink = torch.empty(H, dtype=torch.float32, device=q_s.device) if sink is not None else None
    nbytes = lib.algx_qknorm_attn_bwd_packed_workspace_size(B, H, T, D, dt)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q_s.device)
    L.check(lib.algx_qknorm_attn_bwd_packed(cfg, qkv.data_ptr(), gain_q.data_ptr(), gain_k.data_ptr(),
                                            *_rot_args(rotary), q_s.data_ptr(), k_n.data_ptr(), v_h.data_ptr(),
                                            L.ptr(sink), guard.data_ptr(), o.data_ptr(), L.ptr(o_prec),
                                            stat.data_ptr(), do.data_ptr(), dqkv.data_ptr(), dgq.data_ptr(),
                                            dgk.data_ptr(), L.ptr(dsink), B, H, T, D, dt, float(eps), ws.data_ptr(),
                                            nbytes, st), "algx_qknorm_attn_bwd_packed")
    return dqkv, dgq, dgk, dsink


class _QKNormFlashPacked(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, gain_q, gain_k, sink, cfg: L.AttnConfig, eps: float, rotary):
        o, saved = qknorm_attn_forward_packed(qkv, gain_q, gain_k, sink, cfg, eps, rotary)
        ctx.cfg, ctx.eps, ctx.rotary = cfg, eps, rotary
        ctx.save_for_backward(qkv, gain_q, gain_k, *saved)
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, gain_q, gain_k, *saved = ctx.saved_tensors
        dqkv, dgq, dgk, dsink = qknorm_attn_backward_packed(qkv, gain_q, gain_k, saved, ctx.cfg, do, ctx.eps,
                                                            rotary=ctx.rotary)
        return dqkv, dgq, dgk, dsink, None, None, None


def qknorm_flash_attention_packed(qkv, gain_q, gain_k, sink_logit=None, *, eps: float = 1e-5, kind: str = "asinh",
                                  n: int = 16, c: float = 16.0, block: int = 512, range_guard: bool = False,
                                  shift: Optional[bool] = None, fast_rho: Optional[bool] = None,
                                  inv_stat: Optional[bool] = None, rotary=None):
    """:func:`qknorm_flash_attention` on the token-major output of one QKV
    projection: ``qkv`` (B, T, 3, H, D) holds [q | k | v] per token; returns
    the attention output token-major (B, T, H, D), ready for the output
    projection (model.py:166-180 without the transposes). Same values and
    gradients as transposing q, k, v to (B, H, T, D), calling
    :func:`qknorm_flash_attention` and transposing back."""
    if qkv.ndim != 5 or qkv.shape[2] != 3:
        raise ValueError(f"qkv must have shape (B, T, 3, H, D), got {tuple(qkv.shape)}")
    qkv = qkv.contiguous()
    q_view = qkv[:, :, 0].permute(0, 2, 1, 3)  # shapes and dtypes for validation only
    cfg, sink, gq, gk = qknorm_call_args(q_view, q_view, q_view, gain_q, gain_k, sink_logit, eps, kind, n, c, block,
                                         range_guard, shift, fast_rho, inv_stat)
    rot = rotary_tables(rotary, q_view)
    return _QKNormFlashPacked.apply(qkv, gq, gk, sink, cfg, float(eps), rot)
