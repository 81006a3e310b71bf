"""Fused tied-embedding projection + likelihood (drop-in for kernels/fused_head.py).

``fused_head(h, embed, targets, kind=..., n=..., c=..., block_n=..., block_v=...)``
returns ``(objective, telemetry)`` exactly as the reference (fused_head.py:260-275):
for ``"ce"`` the mean cross-entropy and the per-token NLL; for ``"alg_ce"`` the
mean target-miss probability (whose gradient is the exact log-likelihood
gradient) and the per-token target probability. Telemetry carries no gradient.

Label handling follows the reference kernel's ``col == target`` compare: a
label outside [0, V) matches no column (its target logit is 0) and still
counts in the mean. ``ignore_index`` (an extension, default None) removes rows
whose label equals it from the objective, the gradients and the mean; their
telemetry is 0, and any other label outside [0, V) raises the device error
word (read with ``algx._lib.device_error()``).

The GEMMs run on tcgen05 tensor cores in bfloat16 (``embed`` is cast to the
compute dtype as fused_head.py:168 does; float32 ``h`` is rounded to bfloat16,
which is what a TPU matmul at default precision does with float32 operands).
"""

from __future__ import annotations

import torch

from .. import _lib as L


# The objective's constants and argument checks live in the torch-free
# algx.variants (shared with the JAX front-end); re-exported here.
from ..variants import check_head_options, head_config_lists, head_slope  # noqa: E402,F401


def head_config_from_lists(ints, floats) -> L.HeadConfig:
    """Pack :func:`head_config_lists` into the C ABI's ``AlgxHeadConfig``."""
    cfg = L.HeadConfig()
    cfg.kind, cfg.n, cfg.has_ignore, cfg.ignore_index = (int(i) for i in ints)
    cfg.inv_c, cfg.clamp = (float(f) for f in floats[:2])
    return cfg


def head_config(kind: str, n: int, c: float, vocab: int, ignore_index=None) -> L.HeadConfig:
    return head_config_from_lists(*head_config_lists(kind, n, c, vocab, ignore_index))


def head_forward_partials(h16, e16, t32, cfg, vocab_offset=0):
    """Per-token (m, l, zt) over this embedding shard (fwd kernel + split reduce)."""
    N, d = h16.shape
    V = e16.shape[0]
    lib = L.lib()
    st = L.stream_of(h16)
    splits = lib.algx_head_fwd_splits(N, V)
    part = torch.empty((3, splits, N), dtype=torch.float32, device=h16.device)
    L.check(lib.algx_head_fwd(cfg, h16.data_ptr(), e16.data_ptr(), t32.data_ptr(), part[0].data_ptr(),
                              part[1].data_ptr(), part[2].data_ptr(), N, d, V, vocab_offset, splits, L.ALGX_BF16,
                              st), "algx_head_fwd")
    mlz = torch.empty((3, N), dtype=torch.float32, device=h16.device)
    L.check(lib.algx_head_reduce(cfg, part[0].data_ptr(), part[1].data_ptr(), part[2].data_ptr(), splits, N,
                                 mlz[0].data_ptr(), mlz[1].data_ptr(), mlz[2].data_ptr(), st), "algx_head_reduce")
    return mlz


def head_finalize(cfg, t32, mlz, vocab_total):
    """(stat, telemetry, objective[1], count[1]) from combined statistics."""
    N = t32.shape[0]
    # Four separate tensors (no views of one buffer), so the custom operator
    # front-end can return them without aliasing.
    stat, tel = (torch.empty(N, dtype=torch.float32, device=t32.device) for _ in range(2))
    obj, count = (torch.empty(1, dtype=torch.float32, device=t32.device) for _ in range(2))
    L.check(L.lib().algx_head_finalize(cfg, t32.data_ptr(), mlz[0].data_ptr(), mlz[1].data_ptr(),
                                       mlz[2].data_ptr(), N, vocab_total, stat.data_ptr(), tel.data_ptr(),
                                       obj.data_ptr(), count.data_ptr(), L.stream_of(t32)),
            "algx_head_finalize")
    return stat, tel, obj, count


def head_backward(h16, e16, t32, stat, scale, cfg, vocab_offset=0, dh_dtype=torch.bfloat16, workspace=None):
    """(dh, dembed fp32) for this shard; ``scale`` is a 1-element device tensor.

    ``workspace`` (uint8, at least ``algx_head_bwd_workspace_size`` bytes)
    holds one bf16 logit-gradient slab; it is allocated here when not given.
    """
    N, d = h16.shape
    V = e16.shape[0]
    lib = L.lib()
    code = L.dtype_code(dh_dtype)
    need = lib.algx_head_bwd_workspace_size(N, d, V, code)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=h16.device)
    dh = torch.empty((N, d), dtype=dh_dtype, device=h16.device)
    de = torch.empty((V, d), dtype=torch.float32, device=h16.device)
    L.check(lib.algx_head_bwd(cfg, h16.data_ptr(), e16.data_ptr(), t32.data_ptr(), stat.data_ptr(),
                              scale.data_ptr(), dh.data_ptr(), code, de.data_ptr(), N, d, V, vocab_offset,
                              L.ALGX_BF16, workspace.data_ptr(), workspace.numel(), L.stream_of(h16)),
            "algx_head_bwd")
    return dh, de


class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, embed, targets, cfg, slope):
        h16 = h.to(torch.bfloat16).contiguous()
        e16 = embed.to(torch.bfloat16).contiguous()
        t32 = targets.to(torch.int32).contiguous()
        mlz = head_forward_partials(h16, e16, t32, cfg)
        stat, tel, obj, count = head_finalize(cfg, t32, mlz, e16.shape[0])
        ctx.save_for_backward(h16, e16, t32, stat, count)
        ctx.cfg, ctx.slope = cfg, slope
        ctx.h_dtype, ctx.e_dtype = h.dtype, embed.dtype
        ctx.mark_non_differentiable(tel)
        return obj.reshape(()), tel

    @staticmethod
    def backward(ctx, g_obj, g_tel):
        h16, e16, t32, stat, count = ctx.saved_tensors
        scale = (g_obj.reshape(1).float() * ctx.slope / count).contiguous()
        dh, de = head_backward(h16, e16, t32, stat, scale, ctx.cfg)
        return dh.to(ctx.h_dtype), de.to(ctx.e_dtype), None, None, None


def fused_head(h, embed, targets, *, kind="ce", n=16, c=16.0, block_n=128, block_v=512, ignore_index=None):
    """Fused tied-embedding projection and likelihood objective (kernels/fused_head.py:260-275).

    ``h`` (N, d), ``embed`` (V, d), ``targets`` (N,). Returns ``(objective,
    telemetry)``. ``block_n``/``block_v`` are validated as the reference does
    (N divisible by min(block_n, N)) and do not change the result.
    """
    N, d = check_head_options(kind, n, h.shape, block_n)
    if embed.shape[1] != d or targets.shape != (N,):
        raise ValueError("h (N, d), embed (V, d) and targets (N,) shapes disagree")
    L.require_cuda(h, embed, targets)
    cfg = head_config(kind, n, c, embed.shape[0], ignore_index)
    slope = head_slope(kind, n, c)
    obj, tel = _Head.apply(h, embed, targets, cfg, slope)
    return obj, tel.detach()
