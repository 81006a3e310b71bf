"""Parity at the full headline shapes: BASELINE config 2 (B8 H12 S2048 D64) and
the 350M attention shape of config 4 (B8 H16), bf16, QK-norm -> guarded asinh
attention n=16 c=8, forward and backward.

At these shapes the persistent tcgen05 backward hands each CTA ten or more
(head, key tile) work items, so the paths that only show up across items run:
both K buffers, every slot of the item queue, mbarrier parities carried from
one item to the next, a query ring that wraps across items, and dQ reduce-adds
from many items into one accumulator. The forward runs several waves of CTAs.

A third case raises the QK-norm gains so that the range guard takes the
shifted branch over the whole batch.

Checks, in the spirit of the reference's whole-head test
(tests/test_flash_kernel_tpu.py:253-328, head_resident.py:95-132):

* every head against the shifted CUDA-core kernels (the same function through
  a different code path and rounding), at the bf16 bar of 2e-2;
* a sample of heads against the float64 oracle, head by head (heads are
  independent, so each sampled head is a complete check of its items);
* a second backward with the upstream gradient zero outside the sampled
  heads: the other heads' gradients must be exactly zero, the sampled heads'
  dk and dv bit-identical to the first run, and the gain (and sink)
  gradients, which sum over all heads, equal to the oracle's sum over the
  sampled heads.
"""

import numpy as np
import pytest
import torch

from algx import _lib as L
from algx.kernels import flash as F
from oracle import reference_math as R
from tests.gpu_util import dump, rel_l2

pytestmark = pytest.mark.gpu

T, D, N_POW, C_SCALE, EPS = 2048, 64, 16, 8.0, 1e-5
TOL = 2e-2  # BASELINE bf16 I/O with fp32 accumulation


def _inputs(B, H, with_sink, seed, gain):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn((B, H, T, D), generator=g).to(torch.bfloat16) for _ in range(4))
    gq = gain + 0.02 * torch.randn(D, generator=g)
    gk = gain + 0.02 * torch.randn(D, generator=g)
    sink = 0.5 * torch.randn(H, generator=g) if with_sink else None
    return q, k, v, do, gq, gk, sink


def _run(q, k, v, do, gq, gk, sink, **opts):
    leaves = [t.cuda().requires_grad_(True) for t in (q, k, v)]
    gains = [t.cuda().requires_grad_(True) for t in (gq, gk)]
    s = None if sink is None else sink.cuda().requires_grad_(True)
    o = F.qknorm_flash_attention(*leaves, *gains, s, eps=EPS, kind="asinh", n=N_POW, c=C_SCALE, **opts)
    torch.sum(o.float() * do.cuda().float()).backward()
    torch.cuda.synchronize()
    grads = [t.grad for t in leaves + gains] + [None if s is None else s.grad]
    return o.detach(), grads


def _oracle_head(qh, kh, vh, doh, gq, gk, sink_h):
    """Float64 oracle of one head (1, 1, T, D): rms_norm -> flash_attention, bf16 rounding points."""
    io = torch.bfloat16
    leaves = [t.double().reshape(1, 1, T, D).requires_grad_(True) for t in (qh, kh, vh)]
    gains = [t.double().requires_grad_(True) for t in (gq, gk)]
    s = None if sink_h is None else sink_h.double().reshape(1).requires_grad_(True)
    o = R.flash_attention(R.rms_norm(leaves[0], gains[0], EPS, io), R.rms_norm(leaves[1], gains[1], EPS, io),
                          leaves[2], s, kind="asinh", n=N_POW, c=C_SCALE, range_guard=True, io_dtype=io)
    torch.sum(o * doh.double().reshape(1, 1, T, D)).backward()
    return (o.detach().reshape(T, D), *(t.grad.reshape(T, D) for t in leaves),
            *(t.grad for t in gains), None if s is None else s.grad)


@pytest.mark.parametrize("B,H,with_sink,gain,sample", [
    (8, 12, False, 1.0, (0, 13, 27, 40, 55, 68, 81, 95)),
    (8, 16, True, 1.0, (0, 17, 35, 50, 69, 86, 103, 127)),
    (8, 12, True, 4.5, (1, 14, 30, 47, 58, 70, 83, 94)),
], ids=["config2", "config4_350m_sink", "config2_sink_shifted"])
def test_fullsize_qknorm_attention(B, H, with_sink, gain, sample):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    items = B * H * (T // 128)
    assert items > 2 * sms, "the shape must give every backward CTA several work items"
    q, k, v, do, gq, gk, sink = _inputs(B, H, with_sink, seed=2048 + H, gain=gain)

    # gain 1: the guard chooses the unshifted branch; gain 4.5 puts the
    # product of the squared norms (which grows with gain^4) above the
    # guard's bound of about 251: the shifted branch, which also runs
    # on the tcgen05 kernels under the range guard
    var = F.make_variant("asinh", N_POW, C_SCALE, T)
    sk = F.check_inputs(q.cuda(), k.cuda(), v.cuda(), sink, "asinh", C_SCALE)
    cfg = F.build_config("asinh", var, T, D, C_SCALE, with_sink, True)
    _, _, guard = F.qknorm_attn_prepare(q.cuda(), k.cuda(), v.cuda(), gq.cuda(), gk.cuda(), sk, cfg, EPS)
    m = guard.cpu().tolist()
    low = m[0] * m[1] <= cfg.guard_qk and m[2] <= cfg.guard_v and (not with_sink or m[3] <= cfg.guard_sink)
    assert low == (gain == 1.0), (m, gain)

    L.device_error()  # clear the device error word
    o1, g1 = _run(q, k, v, do, gq, gk, sink, range_guard=True)
    assert L.device_error() == 0

    # every head against the shifted CUDA-core path of the same function
    o_ref, g_ref = _run(q, k, v, do, gq, gk, sink, shift=True)
    assert rel_l2(o1, o_ref) < TOL
    for name, a, b in zip(("dq", "dk", "dv", "dgain_q", "dgain_k", "dsink"), g1, g_ref):
        if b is None:
            continue
        if a.ndim == 4:  # head by head, so one corrupted head cannot hide in the total
            ha, hb = a.reshape(B * H, -1), b.reshape(B * H, -1)
            worst = max(rel_l2(ha[i], hb[i]) for i in range(B * H))
            assert worst < TOL, (name, worst)
        else:
            assert rel_l2(a, b) < TOL, name

    # upstream gradient zero outside the sampled heads
    mask = torch.zeros(B * H, dtype=torch.bool)
    mask[list(sample)] = True
    do_m = (do.reshape(B * H, T, D) * mask[:, None, None].to(do.dtype)).reshape(B, H, T, D)
    o2, g2 = _run(q, k, v, do_m, gq, gk, sink, range_guard=True)
    assert torch.equal(o1, o2)
    for name, a1, a2 in zip(("dq", "dk", "dv"), g1[:3], g2[:3]):
        h1, h2 = a1.reshape(B * H, T, D), a2.reshape(B * H, T, D)
        assert torch.count_nonzero(h2[~mask.cuda()]) == 0, name
        if name != "dq":  # dq goes through reduce-adds whose order varies between calls
            assert torch.equal(h1[mask.cuda()], h2[mask.cuda()]), name

    sum_gq = torch.zeros(D, dtype=torch.float64)
    sum_gk = torch.zeros(D, dtype=torch.float64)
    sum_sink = torch.zeros(H, dtype=torch.float64)
    for bh in sample:
        b, h = divmod(bh, H)
        want = _oracle_head(q[b, h], k[b, h], v[b, h], do[b, h], gq, gk, None if sink is None else sink[h:h + 1])
        got = (o1[b, h], g1[0][b, h], g1[1][b, h], g1[2][b, h])
        for name, a, w in zip(("o", "dq", "dk", "dv"), got, want[:4]):
            err = rel_l2(a, w)
            if err >= TOL:
                dump(f"fullsize_B{B}H{H}_head{bh}_{name}", got=a, want=w)
            assert err < TOL, (bh, name, err)
        sum_gq += want[4]
        sum_gk += want[5]
        if sink is not None:
            sum_sink[h] += float(want[6])
    assert rel_l2(g2[3], sum_gq) < TOL
    assert rel_l2(g2[4], sum_gk) < TOL
    if sink is not None:
        touched = sorted({bh % H for bh in sample})
        assert rel_l2(g2[5][touched], sum_sink[touched]) < TOL
        untouched = [h for h in range(H) if h not in touched]
        assert torch.count_nonzero(g2[5][untouched]) == 0
    assert L.device_error() == 0
