"""Attention kernels vs the float64 oracle.

Cases and tolerances port tests/test_flash_kernel_tpu.py of the reference
(file:line cited per test), plus the golden fixtures made from the
reference's own dense code and the fp32 bar of 1e-3 relative.
"""

import math
import os
from functools import partial

import numpy as np
import pytest
import torch

from algx.kernels.flash import flash_attention
from oracle import reference_math as R
from tests.golden import cases
from tests.gpu_util import algx_attention, dump, oracle_attention, rel_l2

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_dense.npz"))

CASES = [("asinh", 16, 16.0, True, True, False), ("asinh", 16, 16.0, True, True, True),
         ("asinh", 16, 16.0, True, False, True), ("asinh", 16, 16.0, False, False, True),
         ("asinh", 8, 1.0, True, True, False), ("asinh", 32, 8.0, False, True, True)]


def _randn(seed, shape, dtype=torch.float32, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


@pytest.mark.parametrize("kind,n,c,with_sink,shift,fast", CASES)
@pytest.mark.parametrize("block", [128, 256])
def test_flash_matches_dense(kind, n, c, with_sink, shift, fast, block):
    """test_flash_kernel_tpu.py:38-66 (fp32, atol/rtol 2e-3, grads 3e-3 max-normalised)."""
    B, H, T, D = 2, 3, 512, 64
    q = _randn(1, (B, H, T, D), scale=1.5)
    k = _randn(2, (B, H, T, D), scale=1.5)
    v = _randn(3, (B, H, T, D))
    g = _randn(4, (B, H, T, D))
    sink = (_randn(5, (H,)) * 0.5).reshape(1, H, 1, 1) if with_sink else None
    fn = partial(flash_attention, kind=kind, n=n, c=c, block=block, shift=shift, fast_rho=fast)
    got = algx_attention(fn, *(t.cuda() for t in (q, k, v, g)), None if sink is None else sink.cuda())
    want = R.attention_grads(lambda a, b, c_, s: R.asinh_attention(a, b, c_, n=n, c=c, sink_logit=s),
                             q.double(), k.double(), v.double(), g.double(),
                             None if sink is None else sink.double())
    np.testing.assert_allclose(got[0].cpu().double(), want[0], atol=2e-3, rtol=2e-3)
    for a, b in zip(got[1:], want[1:]):
        if b is None:
            continue
        scale = float(b.abs().max()) + 1e-6
        np.testing.assert_allclose(a.cpu().double() / scale, b / scale, atol=3e-3)


@pytest.mark.parametrize("mode", ["root", "inverse", "compact", "guarded", "polynomial"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_model_attention_statistics(mode, dtype):
    """test_flash_kernel_tpu.py:69-97 (n=16, c=8, learned sink; bf16 rel-L2 .02, fp32 .005)."""
    shape = (1, 2, 512, 64)
    q, k, v, g = (_randn(13 + i, shape, dtype) for i in range(4))
    sink = _randn(17, (1, 2, 1, 1))
    fn = partial(flash_attention, kind="asinh", n=16, c=8., shift=False, fast_rho=True,
                 inv_stat=mode != "root", compact_stat=mode in ("compact", "guarded"),
                 range_guard=mode == "guarded", poly_rho=mode == "polynomial")
    got = algx_attention(fn, *(t.cuda() for t in (q, k, v, g)), sink.cuda())
    io = None if dtype == torch.float32 else torch.bfloat16
    want = oracle_attention(q, k, v, g, sink, io_dtype=io, kind="asinh", n=16, c=8.,
                            range_guard=mode == "guarded", shift=False)
    np.testing.assert_allclose(got[0].float().cpu(), want[0].float(), atol=.012, rtol=.012)
    lim = .02 if dtype == torch.bfloat16 else .005
    for name, a, b in zip(("dq", "dk", "dv", "dsink"), got[1:], want[1:]):
        assert rel_l2(a, b) < lim, name


@pytest.mark.parametrize("score_sign", [-1., 1.])
@pytest.mark.parametrize("with_sink", [False, True])
@pytest.mark.parametrize("magnitude", [1000., 1e7])
def test_guarded_attention_tail(score_sign, with_sink, magnitude):
    """test_flash_kernel_tpu.py:100-119: the guard falls back to the shifted branch."""
    shape = (1, 1, 256, 64)
    q = torch.full(shape, math.sqrt(magnitude))
    k = q * score_sign
    v = _randn(29, shape)
    g = torch.ones(shape)
    sink = torch.zeros((1,)) if with_sink else None
    fn = partial(flash_attention, kind="asinh", n=16, c=8., block=128, compact_stat=True, range_guard=True)
    got = algx_attention(fn, q.cuda(), k.cuda(), v.cuda(), g.cuda(), None if sink is None else sink.cuda())
    assert torch.isfinite(got[0]).all()
    want = R.asinh_attention(q.double(), k.double(), v.double(), n=16, c=8.,
                             sink_logit=None if sink is None else sink.double())
    np.testing.assert_allclose(got[0].cpu().double(), want, atol=2e-3, rtol=2e-3)
    for t in got[1:4]:
        assert torch.isfinite(t).all()


def test_explicit_clipping_vjp_is_zero_above_cap():
    """test_flash_kernel_tpu.py:122-138: the clipped primal is flat above the clamp."""
    shape = (1, 1, 256, 64)
    q = torch.full(shape, math.sqrt(1000)).cuda()
    v = _randn(39, shape).cuda()
    g = _randn(40, shape).cuda()
    sink = torch.full((1,), 1000.).cuda()
    fn = partial(flash_attention, kind="asinh", n=16, c=8., block=128, shift=False, range_guard=False)
    _, dq, dk, _, ds = algx_attention(fn, q, q.clone(), v, g, sink)
    for t in (dq, dk, ds):
        assert torch.count_nonzero(t) == 0


@pytest.mark.parametrize("mode", ["sink", "no_sink", "negative", "gain_two", "positive_tail", "negative_tail"])
def test_whole_head_model_shape(mode):
    """test_flash_kernel_tpu.py:253-328: T=2048 bf16 model shape, guarded (rel-L2 .025)."""
    shape = (1, 2, 2048, 64)
    q, k, v, g = (_randn(563 + i, shape, torch.bfloat16) for i in range(4))
    sink = torch.tensor([-.35, .125]).reshape(1, 2, 1, 1)
    if mode in ("no_sink", "negative"):
        sink = None
    if mode == "negative":
        q = (1 + .05 * q.float()).to(torch.bfloat16)
        k = (-1 + .05 * k.float()).to(torch.bfloat16)
    if mode == "gain_two":
        q = (2 * R.rms_norm(q.double(), None, 1e-5, io_dtype=torch.bfloat16)).to(torch.bfloat16)
        k = (2 * R.rms_norm(k.double(), None, 1e-5, io_dtype=torch.bfloat16)).to(torch.bfloat16)
    if mode.endswith("tail"):
        q = torch.full(shape, math.sqrt(1000)).to(torch.bfloat16)
        k = q if mode == "positive_tail" else -q
    fn = partial(flash_attention, kind="asinh", n=16, c=8., range_guard=True)
    got = algx_attention(fn, *(t.cuda() for t in (q, k, v, g)), None if sink is None else sink.cuda())
    io = None if mode.endswith("tail") else torch.bfloat16
    want = oracle_attention(q, k, v, g, sink, io_dtype=io, kind="asinh", n=16, c=8., range_guard=True)
    np.testing.assert_allclose(got[0].float().cpu(), want[0].float(), atol=.015, rtol=.015)
    err2 = norm2 = 0.0
    for idx, (a, b) in enumerate(zip(got[1:], want[1:])):
        if b is None:
            continue
        assert torch.isfinite(a).all()
        a64, b64 = a.double().cpu(), b.double()
        err2 += float(torch.sum((a64 - b64) ** 2))
        norm2 += float(torch.sum(b64 ** 2))
        if mode == "positive_tail" and idx == 0:
            # Equal keys: dQ vanishes up to the rounding of the centred score
            # VJP; bound it by u*sum|ds| as test_flash_kernel_tpu.py:295-314 does.
            va, ga = v.double().numpy(), g.double().numpy()
            count = np.arange(1, shape[-2] + 1, dtype=np.float64)
            ideal = np.cumsum(va, axis=-2) / count[None, None, :, None]
            centered = np.sum(ga * ideal, axis=-1)
            dp = ga @ np.swapaxes(va, -1, -2)
            visible = np.tril(np.ones((shape[-2], shape[-2]), bool))
            mean_abs = np.sum(np.where(visible, np.abs(dp - centered[..., None]), 0.), axis=-1) / count
            kval = float(k[0, 0, 0, 0])
            x = shape[-1] * kval * kval / (8 * math.sqrt(shape[-1]))
            factor = (16 / (8 * math.sqrt(shape[-1]))) * abs(kval) / math.sqrt(1 + x * x)
            roundoff = (2 ** -8 + shape[-2] * 2 ** -24) * (1 + 2 ** -8)
            bound = factor * roundoff * mean_abs + 2e-6
            assert np.all(np.abs(a64.numpy() - b64.numpy()) <= bound[..., None])
        elif mode != "negative":
            assert rel_l2(a64, b64) < .025, idx
    assert math.sqrt(err2 / max(norm2, 1e-12)) < .025


@pytest.mark.parametrize("case", cases.ATTN_CASES, ids=[c[0] for c in cases.ATTN_CASES])
@pytest.mark.parametrize("prec", ["f64", "bf16"])
def test_against_reference_goldens(case, prec):
    """Kernel vs outputs of the reference's own dense code (tests/golden)."""
    name, n, c, with_sink, scale = case
    idx = cases.ATTN_CASES.index(case)
    q, k, v, g, sink = cases.attn_inputs(100 + 10 * idx, scale=scale, with_sink=with_sink)
    dt = torch.float32 if prec == "f64" else torch.bfloat16
    t = [torch.from_numpy(a).to(dt).cuda() for a in (q, k, v)]
    gg = torch.from_numpy(g).cuda()
    s = None if sink is None else torch.from_numpy(sink).cuda()
    fn = partial(flash_attention, kind="asinh", n=n, c=c, range_guard=True)
    got = algx_attention(fn, *t, gg, s)
    key = f"attn_{name}_{prec}"
    tol = 1e-3 if prec == "f64" else 2e-2
    names = ["o", "dq", "dk", "dv"] + (["dsink"] if with_sink else [])
    for nm, a in zip(names, got):
        err = rel_l2(a, torch.from_numpy(GOLD[f"{key}_{nm}"]))
        if err >= tol:
            dump(f"golden_{key}_{nm}", got=a, want=GOLD[f"{key}_{nm}"])
        assert err < tol, (nm, err)


def test_baseline_config1_qknorm_then_attention():
    """The CPU-runnable configuration: B2 H4 S512 D64 fp32, QK-norm (gain 1) then guarded asinh n16 c8.

    The fp32 bar of the north star: outputs and grads within 1e-3 relative.
    """
    from algx.kernels.qk_norm import qk_rms_norm
    shape = (2, 4, 512, 64)
    q, k, v = (_randn(i, shape) for i in (0, 10, 20))
    do = _randn(1, shape)
    gain = torch.ones(64)
    leaves = [t.cuda().requires_grad_(True) for t in (q, k, v)]
    gq = gain.cuda().requires_grad_(True)
    gk = gain.cuda().requires_grad_(True)
    o = flash_attention(qk_rms_norm(leaves[0], gq), qk_rms_norm(leaves[1], gk), leaves[2],
                        kind="asinh", n=16, c=8., range_guard=True)
    torch.sum(o * do.cuda()).backward()
    ref_leaves = [t.double().requires_grad_(True) for t in (q, k, v)]
    rq = gain.double().requires_grad_(True)
    rk = gain.double().requires_grad_(True)
    ro = R.flash_attention(R.rms_norm(ref_leaves[0], rq), R.rms_norm(ref_leaves[1], rk), ref_leaves[2],
                           kind="asinh", n=16, c=8., range_guard=True)
    torch.sum(ro * do.double()).backward()
    assert rel_l2(o.detach(), ro.detach()) < 1e-3
    for a, b in zip([*leaves, gq, gk], [*ref_leaves, rq, rk]):
        assert rel_l2(a.grad, b.grad) < 1e-3


@pytest.mark.parametrize("T", [128, 256, 1024])
@pytest.mark.parametrize("n,c", [(16, 8.0), (8, 2.0), (32, 8.0)])
def test_fast_path_shapes(T, n, c):
    """tcgen05 path (bf16, T % 128 == 0) at single-tile, two-tile and longer rows."""
    from algx import _lib as L
    shape = (2, 3, T, 64)
    q, k, v, g = (_randn(700 + i + T, shape, torch.bfloat16) for i in range(4))
    sink = _randn(7, (3,)) * 0.3
    fn = partial(flash_attention, kind="asinh", n=n, c=c, range_guard=True)
    got = algx_attention(fn, *(t.cuda() for t in (q, k, v, g)), sink.cuda())
    assert L.device_error() == 0
    want = oracle_attention(q, k, v, g, sink, io_dtype=torch.bfloat16, kind="asinh", n=n, c=c, range_guard=True)
    np.testing.assert_allclose(got[0].float().cpu(), want[0].float(), atol=.015, rtol=.015)
    for name, a, b in zip(("dq", "dk", "dv", "dsink"), got[1:], want[1:]):
        err = rel_l2(a, b)
        if err >= .025:
            dump(f"fast_T{T}_n{n}_{name}", got=a, want=b)
        assert err < .025, (name, err)


@pytest.mark.parametrize("dtype,with_sink", [(torch.bfloat16, False), (torch.bfloat16, True), (torch.float32, False)])
def test_fused_qknorm_prologue_matches_composed(dtype, with_sink):
    """qknorm_flash_attention == flash_attention(qk_rms_norm(q), qk_rms_norm(k), v) (model.py:170-174).

    The fused prologue goes through the same rounding points, so the output is
    bit-identical; gradients agree up to the order of the dQ reduce-adds.
    """
    from algx.kernels.flash import qknorm_flash_attention
    from algx.kernels.qk_norm import qk_rms_norm
    shape = (2, 3, 512, 64)
    q, k, v, do = (_randn(40 + i, shape, dtype) for i in range(4))
    gq0, gk0 = 1 + 0.02 * _randn(50, (64,)), 1 + 0.02 * _randn(51, (64,))
    sink0 = _randn(52, (3,)) if with_sink else None

    def run(fused):
        leaves = [t.cuda().requires_grad_(True) for t in (q, k, v)]
        gains = [g.cuda().requires_grad_(True) for g in (gq0, gk0)]
        sink = sink0.cuda().requires_grad_(True) if with_sink else None
        opts = dict(kind="asinh", n=16, c=8., range_guard=True)
        if fused:
            o = qknorm_flash_attention(*leaves, *gains, sink, eps=1e-5, **opts)
        else:
            o = flash_attention(qk_rms_norm(leaves[0], gains[0]), qk_rms_norm(leaves[1], gains[1]), leaves[2],
                                sink, **opts)
        torch.sum(o.float() * do.cuda().float()).backward()
        grads = [t.grad for t in leaves + gains] + ([sink.grad] if with_sink else [])
        return o.detach(), grads

    o_f, g_f = run(True)
    o_c, g_c = run(False)
    assert torch.equal(o_f, o_c)
    lim = 1e-2 if dtype == torch.bfloat16 else 1e-5
    for a, b in zip(g_f, g_c):
        assert rel_l2(a, b) < lim


@pytest.mark.parametrize("dtype,guard,gain,with_sink", [
    (torch.bfloat16, True, 1., False), (torch.bfloat16, True, 1., True), (torch.bfloat16, True, 20., True),
    (torch.bfloat16, False, 1., False), (torch.float32, True, 1., True)])
def test_fused_qknorm_backward_matches_composed(dtype, guard, gain, with_sink):
    """algx_qknorm_attn_bwd == algx_attn_bwd then algx_qknorm_bwd on q and k, on the same residuals.

    gain 20 makes the scores exceed the guard bound, so the guarded mode's
    shifted branch runs (on the tcgen05 backward too, for bf16). dk, dv and
    dsink are computed in a fixed order and must match bit for bit, as must dq
    wherever it does not come from the dQ reduce-adds (whose order varies
    between any two calls: bf16 I/O); dgain differs only by the order of its
    sums.
    """
    from algx.kernels import flash as F
    from algx.kernels.qk_norm import qknorm_backward
    B, H, T, D = 2, 3, 512, 64
    q, k, v, do = (_randn(60 + i, (B, H, T, D), dtype).cuda() for i in range(4))
    gq = (gain + 0.02 * _randn(70, (D,))).cuda()
    gk = (gain + 0.02 * _randn(71, (D,))).cuda()
    sink_logit = _randn(72, (H,)).cuda() if with_sink else None
    var = F.make_variant("asinh", 16, 8., T)
    sink = F.check_inputs(q, k, v, sink_logit, "asinh", 8.)
    cfg = F.build_config("asinh", var, T, D, 8., with_sink, guard)
    o, saved = F.attn_forward_qknorm(q, k, v, gq, gk, sink, cfg, 1e-5)
    fused = F.qknorm_attn_backward(q, k, gq, gk, saved, cfg, do, 1e-5)
    dq, dk, dv, dsink = F.attn_backward(saved, cfg, do)
    dxq, dgq = qknorm_backward(q, gq, dq, 1e-5)
    dxk, dgk = qknorm_backward(k, gk, dk, 1e-5)
    torch.cuda.synchronize()
    g = saved[7].cpu().tolist()  # max||q_s||^2, max||k||^2, max|v|, max|sink| (attn_common.cuh)
    low = g[0] * g[1] <= cfg.guard_qk and g[2] <= cfg.guard_v and (not with_sink or g[3] <= cfg.guard_sink)
    shifted = guard and not low
    fast_dq = dtype == torch.bfloat16  # both branches reduce-add dq on the tcgen05 path
    assert torch.equal(fused[1], dxk) and torch.equal(fused[2], dv)
    if with_sink:
        assert torch.equal(fused[5], dsink)
    if fast_dq:
        assert rel_l2(fused[0], dxq) < 2e-3
    else:
        assert torch.equal(fused[0], dxq)
    for a, b in ((fused[3], dgq), (fused[4], dgk)):
        assert rel_l2(a, b) < (1e-3 if fast_dq else 1e-5)
    if gain == 20.:
        assert shifted, "the large gains should have selected the shifted branch"


def _sharded_vs_single(rank, world, init_file, q_out):
    """Rank r runs batch slice r of a logical batch through the sharded API and
    compares with one single-GPU call on the whole batch (on its own GPU)."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "algebraic-extra_b200")]
    import torch.distributed as dist
    from algx.kernels.flash import qknorm_flash_attention
    from algx.parallel import sharded_qknorm_flash_attention
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        B, H, T, D = 2 * world, 3, 256, 64
        g = torch.Generator().manual_seed(81)
        q, k, v, do = (torch.randn((B, H, T, D), generator=g).to(torch.bfloat16).cuda() for _ in range(4))
        v[-1, 0, 5, 7] = 3e8  # the last slice alone exceeds the guard's max|v|: the shifted branch everywhere
        gq0, gk0 = (1 + 0.02 * torch.randn(64, generator=g)).cuda(), (1 + 0.02 * torch.randn(64, generator=g)).cuda()
        sink0 = torch.randn(H, generator=g).cuda()
        opts = dict(kind="asinh", n=16, c=8., range_guard=True)

        def run(sharded):
            lo = 2 * rank if sharded else 0
            hi = lo + 2 if sharded else B
            leaves = [t[lo:hi].clone().requires_grad_(True) for t in (q, k, v)]
            gains = [x.clone().requires_grad_(True) for x in (gq0, gk0)]
            sink = sink0.clone().requires_grad_(True)
            fn = partial(sharded_qknorm_flash_attention, shard="batch") if sharded else qknorm_flash_attention
            o = fn(*leaves, *gains, sink, **opts)
            torch.sum(o.float() * do[lo:hi].float()).backward()
            return o.detach(), [t.grad for t in leaves], [x.grad for x in gains] + [sink.grad]

        o_s, g_s, shared_s = run(True)
        o_f, g_f, shared_f = run(False)
        sl = slice(2 * rank, 2 * rank + 2)
        ok_o = torch.equal(o_s, o_f[sl])
        ok_g = all(rel_l2(a, b[sl]) < 1e-2 for a, b in zip(g_s, g_f))
        ok_shared = all(rel_l2(a, b) < 1e-3 for a, b in zip(shared_s, shared_f))
        q_out.put((rank, bool(ok_o), bool(ok_g), bool(ok_shared)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_qknorm_attention_two_gpus():
    """Batch split over two GPUs == one call on the whole batch, including the
    range guard's branch (decided on the maxima over both ranks) and the
    summed gain and sink gradients."""
    import tempfile
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        procs = [ctx.Process(target=_sharded_vs_single, args=(r, 2, os.path.join(tmp, "pg"), q_out))
                 for r in range(2)]
        for p in procs:
            p.start()
        results = [q_out.get(timeout=300) for _ in range(2)]
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    for rank, ok_o, ok_g, ok_shared in results:
        assert ok_o and ok_g and ok_shared, (rank, ok_o, ok_g, ok_shared)


def test_sharded_qknorm_attention_one_rank_matches_single():
    """With one rank the sharded entry is the single-GPU entry (same branch, same values)."""
    import tempfile
    import torch.distributed as dist
    from algx.kernels.flash import qknorm_flash_attention
    from algx.parallel import sharded_qknorm_flash_attention
    shape = (2, 3, 256, 64)
    q, k, v, do = (_randn(90 + i, shape, torch.bfloat16).cuda() for i in range(4))
    gq0, gk0 = (1 + 0.02 * _randn(95, (64,))).cuda(), (1 + 0.02 * _randn(96, (64,))).cuda()
    with tempfile.TemporaryDirectory() as tmp:
        dist.init_process_group("nccl", init_method=f"file://{os.path.join(tmp, 'pg')}", rank=0, world_size=1,
                                device_id=torch.device("cuda", torch.cuda.current_device()))
        try:
            outs = []
            for fn in (qknorm_flash_attention, partial(sharded_qknorm_flash_attention, shard="heads")):
                leaves = [t.clone().requires_grad_(True) for t in (q, k, v, gq0, gk0)]
                o = fn(*leaves, kind="asinh", n=16, c=8., range_guard=True)
                torch.sum(o.float() * do.float()).backward()
                outs.append((o.detach(), [t.grad for t in leaves]))
        finally:
            dist.destroy_process_group()
    assert torch.equal(outs[0][0], outs[1][0])
    for a, b in zip(outs[0][1], outs[1][1]):
        assert rel_l2(a, b) < 1e-2


def _torch_rotary(x, cos, sin):
    """The fused prologue's rotation restated with torch ops: tables rounded to
    x's dtype, products and sums in fp32 (separate roundings), one rounding back."""
    half = x.shape[-1] // 2
    t = x.shape[-2]
    c = cos[:t].to(x.dtype).float()
    s = sin[:t].to(x.dtype).float()
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).to(x.dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("table", ["rope", "cayley"])
@pytest.mark.parametrize("with_sink", [False, True])
def test_fused_rotary_prologue_matches_composed(dtype, table, with_sink):
    """qknorm_flash_attention(rotary=...) == flash_attention(rot(qk_rms_norm(q)), rot(qk_rms_norm(k)), v)
    (model.py:170-174): the output bit for bit; gradients up to the order of the dQ reduce-adds."""
    from algx import rotary as P
    from algx.kernels.flash import qknorm_flash_attention
    from algx.kernels.qk_norm import qk_rms_norm
    B, H, T, D = 2, 3, 512, 64
    q, k, v, do = (_randn(110 + i, (B, H, T, D), dtype) for i in range(4))
    gq0, gk0 = 1 + 0.02 * _randn(115, (64,)), 1 + 0.02 * _randn(116, (64,))
    sink0 = _randn(117, (H,)) if with_sink else None
    tabs = P.rope_table(64, 640) if table == "rope" else P.cayley_table_geometric(64, 640)
    tabs = tuple(t.cuda() for t in tabs)

    def run(fused):
        leaves = [t.cuda().requires_grad_(True) for t in (q, k, v)]
        gains = [g.cuda().requires_grad_(True) for g in (gq0, gk0)]
        sink = sink0.cuda().requires_grad_(True) if with_sink else None
        opts = dict(kind="asinh", n=16, c=8., range_guard=True)
        if fused:
            o = qknorm_flash_attention(*leaves, *gains, sink, eps=1e-5, rotary=tabs, **opts)
        else:
            rq = _torch_rotary(qk_rms_norm(leaves[0], gains[0]), *tabs)
            rk = _torch_rotary(qk_rms_norm(leaves[1], gains[1]), *tabs)
            o = flash_attention(rq, rk, leaves[2], sink, **opts)
        torch.sum(o.float() * do.cuda().float()).backward()
        return o.detach(), [t.grad for t in leaves + gains] + ([sink.grad] if with_sink else [])

    o_f, g_f = run(True)
    o_c, g_c = run(False)
    assert torch.equal(o_f, o_c)
    lim = 1e-2 if dtype == torch.bfloat16 else 1e-5
    for a, b in zip(g_f, g_c):
        assert rel_l2(a, b) < lim


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-3), (torch.bfloat16, 2e-2)])
def test_fused_rotary_attention_vs_oracle(dtype, tol):
    """QK-norm -> RoPE -> guarded asinh attention against the float64 oracle
    (rms_norm, apply_rotary, flash_attention of oracle/reference_math.py)."""
    from algx import rotary as P
    from algx.kernels.flash import qknorm_flash_attention
    B, H, T, D = 1, 2, 256, 64
    q, k, v, do = (_randn(120 + i, (B, H, T, D), dtype) for i in range(4))
    gq0 = 1 + 0.02 * _randn(125, (64,))
    gk0 = 1 + 0.02 * _randn(126, (64,))
    cos, sin = P.rope_table(64, T)
    leaves = [t.cuda().requires_grad_(True) for t in (q, k, v, gq0, gk0)]
    o = qknorm_flash_attention(*leaves, kind="asinh", n=16, c=8., range_guard=True, rotary=(cos.cuda(), sin.cuda()))
    torch.sum(o.float() * do.cuda().float()).backward()
    io = None if dtype == torch.float32 else dtype
    ref = [t.double().requires_grad_(True) for t in (q, k, v, gq0, gk0)]
    rq = R.apply_rotary(R.rms_norm(ref[0], ref[3], 1e-5, io), cos.double(), sin.double(), io)
    rk = R.apply_rotary(R.rms_norm(ref[1], ref[4], 1e-5, io), cos.double(), sin.double(), io)
    ro = R.flash_attention(rq, rk, ref[2], kind="asinh", n=16, c=8., range_guard=True, io_dtype=io)
    torch.sum(ro * do.double()).backward()
    assert rel_l2(o.detach(), ro.detach()) < tol
    for a, b in zip(leaves, ref):
        assert rel_l2(a.grad, b.grad) < tol
