"""Vocabulary-parallel head exchange on CPU ranks (gloo, world size 2).

Each rank evaluates its vocabulary slice with the oracle, combines the
per-token statistics with algx.parallel.combine_vocab_stats, and must get the
full-vocabulary statistics; the partial dh all-reduce must give the full dh.
"""

import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _shard_stats(h, e_shard, t, offset, kind, n, c, clamp):
    z = h @ e_shard.T
    cols = torch.arange(e_shard.shape[0])[None, :] + offset
    zt = torch.sum((cols == t[:, None]).to(z.dtype) * z, -1)
    if kind == "ce":
        m = z.max(-1).values
        l = torch.exp(z - m[:, None]).sum(-1)
    else:
        x = torch.minimum(z / c, torch.full_like(z, clamp))
        rad = 1 + x * x
        w = (x + rad * torch.rsqrt(rad)) ** n
        m = torch.zeros(z.shape[0], dtype=z.dtype)
        l = w.sum(-1)
    return torch.stack([m, l, zt])


def _worker(rank, init_file, kind, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "algebraic-extra_b200")]
    from algx.parallel import combine_vocab_stats, shard_rows
    from oracle import reference_math as R
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=WORLD)
    try:
        g = torch.Generator().manual_seed(5)
        N, d, V, n, c = 64, 32, 301, 8, 2.0
        h = torch.randn((N, d), generator=g, dtype=torch.float64)
        e = torch.randn((V, d), generator=g, dtype=torch.float64) * 0.3
        t = torch.randint(0, V, (N,), generator=g)
        clamp = R.likelihood_clamp(V, n)
        off, cnt = shard_rows(V, WORLD, rank)
        mlz = _shard_stats(h, e[off:off + cnt], t, off, kind, n, c, clamp)
        combine_vocab_stats(mlz, kind)
        full = _shard_stats(h, e, t, 0, kind, n, c, clamp)
        if kind == "ce":
            stat, stat_full = mlz[0] + torch.log(mlz[1]), full[0] + torch.log(full[1])
        else:
            stat, stat_full = R.inv_root(mlz[1], n), R.inv_root(full[1], n)
        ok_stat = torch.allclose(stat, stat_full, rtol=1e-12, atol=1e-12)
        ok_zt = torch.allclose(mlz[2], full[2], rtol=1e-12, atol=1e-12)
        # partial dh over the slice, summed across ranks = full dh
        dh_full, _ = R.fused_head_backward(h, e, t, kind=kind, n=n, c=c)
        z = h @ e[off:off + cnt].T
        y = (torch.arange(cnt)[None, :] + off == t[:, None]).to(z.dtype)
        if kind == "ce":
            dz = torch.exp(z - stat[:, None]) - y
            slope = 1.0
        else:
            x = torch.minimum(z / c, torch.full_like(z, clamp))
            rad = 1 + x * x
            r = torch.rsqrt(rad)
            dz = (((x + rad * r) * stat[:, None]) ** n - y) * r
            slope = n / c
        dh = (dz * (slope / N)) @ e[off:off + cnt]
        dist.all_reduce(dh)
        ok_dh = torch.allclose(dh, dh_full, rtol=1e-10, atol=1e-13)
        q.put((rank, bool(ok_stat), bool(ok_zt), bool(ok_dh)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["ce", "alg_ce"])
def test_vocab_parallel_stats_and_dh_allreduce(kind):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init_file = os.path.join(tmp, "pg")
        procs = [ctx.Process(target=_worker, args=(r, init_file, kind, q)) for r in range(WORLD)]
        for p in procs:
            p.start()
        results = [q.get(timeout=120) for _ in range(WORLD)]
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    for rank, ok_stat, ok_zt, ok_dh in results:
        assert ok_stat and ok_zt and ok_dh, (rank, ok_stat, ok_zt, ok_dh)


def test_shard_rows_cover_vocabulary_once():
    from algx.parallel import shard_rows
    for V in (50304, 301, 7):
        for world in (1, 2, 3, 8):
            parts = [shard_rows(V, world, r) for r in range(world)]
            assert parts[0][0] == 0
            assert sum(c for _, c in parts) == V
            for (o1, c1), (o2, _) in zip(parts, parts[1:]):
                assert o1 + c1 == o2


def _guard_worker(rank, init_file, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "algebraic-extra_b200")]
    from algx.parallel import combine_guard, sum_shared_grads
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=WORLD)
    try:
        # per-rank maxima (max||q_s||^2, max||k||^2, max|v|, max|sink|); rank 1 saw a NaN
        mine = [torch.tensor([0.2, 7.0, 1.5, 0.3]), torch.tensor([0.4, float("nan"), 0.5, 0.1])][rank]
        g = combine_guard(mine.clone())
        ok_guard = torch.equal(g, torch.tensor([0.4, float("inf"), 1.5, 0.3]))
        dg = [torch.full((64,), 1.0 + rank, dtype=torch.float32), torch.arange(64, dtype=torch.float32) * rank,
              torch.full((3,), 0.5)]
        s = sum_shared_grads(dg)
        ok_sum = (torch.equal(s[0], torch.full((64,), 3.0)) and torch.equal(s[1], torch.arange(64.0))
                  and torch.equal(s[2], torch.ones(3)) and all(a.shape == b.shape for a, b in zip(s, dg)))
        q.put((rank, bool(ok_guard), bool(ok_sum)))
    finally:
        dist.destroy_process_group()


def test_sharded_attention_guard_and_shared_grads():
    """Sharded attention: the range guard's maxima become global maxima on every rank
    (NaN as +inf, the same shifted-branch decision), and the shared gains'
    gradients are summed over the ranks."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init_file = os.path.join(tmp, "pg")
        procs = [ctx.Process(target=_guard_worker, args=(r, init_file, q)) for r in range(WORLD)]
        for p in procs:
            p.start()
        results = [q.get(timeout=120) for _ in range(WORLD)]
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    for rank, ok_guard, ok_sum in results:
        assert ok_guard and ok_sum, (rank, ok_guard, ok_sum)
