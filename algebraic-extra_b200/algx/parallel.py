"""Multi-GPU pieces of the hot path (one process per GPU, torch.distributed).

* Attention and QK-norm shard by (batch x heads) with no exchange on the data
  path: each rank runs its own slice of one logical batch. For branch parity
  with a single call on the whole batch, the range guard's maxima are
  all-reduced (MAX, 4 floats) between the prologue and the forward kernels,
  and the gradients of the shared parameters (QK-norm gains, and the sink
  when the batch rather than the heads is split) are all-reduced (SUM).
* The fused head is vocabulary-parallel: rank r holds a
  contiguous slice of the embedding rows. The forward computes per-token
  (max, sum, target logit) over the local slice, then all-reduces them
  (one all-gather and a local combine for "ce"; a SUM for the additive
  "alg_ce"); the backward
  computes the local dE slice with no communication and all-reduces the
  partial dh. Collectives go through NCCL on GPU (gloo in the CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib as L
from .kernels import flash as F
from .kernels import fused_head as FH


def shard_rows(total: int, world: int, rank: int):
    """Contiguous split of ``total`` rows over ``world`` ranks: (offset, count)."""
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    offset = rank * base + min(rank, extra)
    return offset, count


def combine_vocab_stats(mlz: torch.Tensor, kind: str, group=None) -> torch.Tensor:
    """Turn per-shard (m, l, zt) rows of ``mlz`` (3, N) into global ones, in place.

    "ce": m_g = max_r m_r, l = sum_r l_r exp(m_r - m_g); "alg_ce": l = sum_r l_r.
    zt is a sum (only the rank owning the target column contributes).
    """
    if kind == "ce":
        # one collective: every rank gathers all ranks' (m, l, zt) and combines
        # them in the same fixed order, so all ranks hold identical statistics
        world = dist.get_world_size(group)
        flat = torch.empty((world * mlz.shape[0],) + tuple(mlz.shape[1:]), dtype=mlz.dtype, device=mlz.device)
        dist.all_gather_into_tensor(flat, mlz.contiguous(), group=group)  # rank blocks stacked along dim 0
        parts = flat.view((world,) + tuple(mlz.shape))
        mg = parts[:, 0].amax(dim=0)
        mlz[1].copy_(torch.sum(parts[:, 1] * torch.exp(parts[:, 0] - mg), dim=0))
        mlz[2].copy_(torch.sum(parts[:, 2], dim=0))
        mlz[0].copy_(mg)
        return mlz
    dist.all_reduce(mlz[1:], op=dist.ReduceOp.SUM, group=group)
    return mlz


class _VocabParallelHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, embed_shard, targets, cfg, slope, kind, vocab_offset, vocab_total, group):
        h16 = h.to(torch.bfloat16).contiguous()
        e16 = embed_shard.to(torch.bfloat16).contiguous()
        t32 = targets.to(torch.int32).contiguous()
        mlz = FH.head_forward_partials(h16, e16, t32, cfg, vocab_offset)
        combine_vocab_stats(mlz, kind, group)
        stat, tel, obj, count = FH.head_finalize(cfg, t32, mlz, vocab_total)
        ctx.save_for_backward(h16, e16, t32, stat, count)
        ctx.cfg, ctx.slope, ctx.voff, ctx.group = cfg, slope, vocab_offset, group
        ctx.h_dtype, ctx.e_dtype = h.dtype, embed_shard.dtype
        ctx.mark_non_differentiable(tel)
        return obj.reshape(()), tel

    @staticmethod
    def backward(ctx, g_obj, g_tel):
        h16, e16, t32, stat, count = ctx.saved_tensors
        scale = (g_obj.reshape(1).float() * ctx.slope / count).contiguous()
        dh, de = FH.head_backward(h16, e16, t32, stat, scale, ctx.cfg, ctx.voff, dh_dtype=torch.float32)
        dist.all_reduce(dh, op=dist.ReduceOp.SUM, group=ctx.group)
        return dh.to(ctx.h_dtype), de.to(ctx.e_dtype), None, None, None, None, None, None, None


def vocab_parallel_fused_head(h, embed_shard, targets, *, vocab_offset: int, vocab_total: int, kind="ce", n=16,
                              c=16.0, ignore_index=None, group=None):
    """``fused_head`` with the embedding rows split over the ranks of ``group``.

    Every rank passes the same ``h`` and ``targets`` and its own slice
    ``embed_shard`` = embed[vocab_offset : vocab_offset + V_local]. Returns the
    same (objective, telemetry) on every rank; gradients: dh (all-reduced) and
    the local slice of dE.
    """
    if kind not in ("ce", "alg_ce"):
        raise ValueError(kind)
    if embed_shard.shape[0] < 1:
        raise ValueError("every rank needs at least one vocabulary row (embed_shard is empty)")
    L.require_cuda(h, embed_shard, targets)
    cfg = FH.head_config(kind, n, c, vocab_total, ignore_index)
    slope = 1.0 if kind == "ce" else n / c
    obj, tel = _VocabParallelHead.apply(h, embed_shard, targets, cfg, slope, kind, vocab_offset, vocab_total,
                                        group)
    return obj, tel.detach()


# ------------------------------------------------------------------ attention
def combine_guard(guard: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's range-guard maxima -> the maxima over all ranks, in place.

    The reference takes them over the whole batch (kernels/flash.py:841-849).
    NaN becomes +inf first: both fail every guard comparison (the shifted
    branch), and a MAX reduction need not propagate NaN.
    """
    torch.nan_to_num_(guard, nan=float("inf"))
    dist.all_reduce(guard, op=dist.ReduceOp.MAX, group=group)
    return guard


def sum_shared_grads(grads, group=None):
    """All-reduce (SUM) a list of gradient tensors as one flat buffer; returns new tensors."""
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    out, i = [], 0
    for g in grads:
        out.append(flat[i:i + g.numel()].view_as(g))
        i += g.numel()
    return out


class _ShardedQKNormFlash(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, gain_q, gain_k, sink, cfg, eps, group, sum_sink, rotary):
        q_s, k_n, guard = F.qknorm_attn_prepare(q, k, v, gain_q, gain_k, sink, cfg, eps, rotary)
        combine_guard(guard, group)
        o, saved = F.attn_forward_prepared(q_s, k_n, v, sink, guard, cfg)
        ctx.cfg, ctx.eps, ctx.group, ctx.sum_sink, ctx.rotary = cfg, eps, group, sum_sink, rotary
        ctx.save_for_backward(q, k, gain_q, gain_k, *saved)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, gain_q, gain_k, *saved = ctx.saved_tensors
        dxq, dxk, dv, dgq, dgk, dsink = F.qknorm_attn_backward(q, k, gain_q, gain_k, saved, ctx.cfg, do, ctx.eps,
                                                               rotary=ctx.rotary)
        shared = [dgq, dgk] + ([dsink] if ctx.sum_sink and dsink is not None else [])
        shared = sum_shared_grads(shared, ctx.group)
        dgq, dgk = shared[0], shared[1]
        if ctx.sum_sink and dsink is not None:
            dsink = shared[2]
        return dxq, dxk, dv, dgq, dgk, dsink, None, None, None, None, None


def sharded_qknorm_flash_attention(q, k, v, gain_q, gain_k, sink_logit=None, *, shard: str = "batch",
                                   group=None, eps: float = 1e-5, kind: str = "asinh", n: int = 16,
                                   c: float = 16.0, block: int = 512, range_guard: bool = False, shift=None,
                                   fast_rho=None, inv_stat=None, rotary=None):
    """``qknorm_flash_attention`` on this rank's slice of one logical batch.

    ``shard="batch"``: every rank holds some of the sequences with all heads,
    and the same ``sink_logit`` (its gradient is summed over the ranks).
    ``shard="heads"``: every rank holds some of the heads of every sequence,
    and the matching slice of ``sink_logit`` (its gradient stays local).
    The QK-norm gains are shared in both cases (their gradients are summed).
    Outputs and gradients equal those of one call on the whole batch, with
    the range guard decided on the maxima over all ranks.
    """
    if shard not in ("batch", "heads"):
        raise ValueError(f"shard must be 'batch' or 'heads', got {shard!r}")
    cfg, sink, gq, gk = F.qknorm_call_args(q, k, v, gain_q, gain_k, sink_logit, eps, kind, n, c, block, range_guard,
                                           shift, fast_rho, inv_stat)
    return _ShardedQKNormFlash.apply(q.contiguous(), k.contiguous(), v.contiguous(), gq, gk, sink, cfg, float(eps),
                                     group, shard == "batch", F.rotary_tables(rotary, q))
