"""Fused head kernels vs the oracle (cases of tests/test_fused_head_tpu.py:13-67, plus ce,
ignore_index, golden fixtures and the benchmark head (N=16384, d=768, V=50304) at full size)."""

import os

import numpy as np
import pytest
import torch

from algx.kernels.fused_head import fused_head
from oracle import reference_math as R
from tests.golden import cases
from tests.gpu_util import rel_l2

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_dense.npz"))


def _inputs(N, d, V, e_scale, seed, ignore_frac=0.0):
    g = torch.Generator().manual_seed(seed)
    h = torch.randn((N, d), generator=g).to(torch.bfloat16)
    e = torch.randn((V, d), generator=g) * e_scale
    t = torch.randint(0, V, (N,), generator=g)
    if ignore_frac:
        t[torch.rand(N, generator=g) < ignore_frac] = -100
    return h, e, t


def _run(h, e, t, **kw):
    hc = h.cuda().requires_grad_(True)
    ec = e.cuda().requires_grad_(True)
    obj, tel = fused_head(hc, ec, t.cuda(), **kw)
    obj.backward()
    torch.cuda.synchronize()
    return obj.detach().cpu(), tel.cpu(), hc.grad.cpu(), ec.grad.cpu()


def _oracle(h, e, t, kind, n, c, ignore_index=None):
    hh, ee = h.double(), e.double()
    obj, tel, _, _ = R.fused_head_forward(hh, ee, t, kind=kind, n=n, c=c, ignore_index=ignore_index,
                                          io_dtype=torch.bfloat16)
    dh, de = R.fused_head_backward(hh, ee, t, kind=kind, n=n, c=c, ignore_index=ignore_index,
                                   io_dtype=torch.bfloat16)
    return obj, tel, dh, de


@pytest.mark.parametrize("kind,n,c", [("alg_ce", 16, 16.0), ("alg_ce", 8, 2.0)])
@pytest.mark.parametrize("V", [32768, 4096])
def test_fused_head_matches_dense(kind, n, c, V):
    """test_fused_head_tpu.py:13-40: objective rtol 2e-3/atol 2e-4, grads cosine > 0.999."""
    h, e, t = _inputs(1024, 256, V, 0.15, 0)
    obj, tel, dh, de = _run(h, e, t, kind=kind, n=n, c=c, block_n=256, block_v=1024)
    o2, t2, dh2, de2 = _oracle(h, e, t, kind, n, c)
    np.testing.assert_allclose(obj.item(), o2.item(), rtol=2e-3, atol=2e-4)
    np.testing.assert_allclose(tel.double(), t2, rtol=2e-2, atol=2e-4)
    for a, b in ((dh, dh2), (de, de2)):
        a, b = a.double(), b.double()
        scale = float(b.abs().max()) + 1e-12
        np.testing.assert_allclose(a / scale, b / scale, atol=2e-2)
        cos = float((a * b).sum() / torch.sqrt((a * a).sum() * (b * b).sum()))
        assert cos > 0.999


@pytest.mark.parametrize("width", [768, 1024])
def test_production_head_tiles_at_model_widths(width):
    """test_fused_head_tpu.py:43-67: alg_ce n=8 c=2, V=32768, grads rel-L2 < 1e-2."""
    h, e, t = _inputs(256, width, 32768, 0.02, 42)
    obj, tel, dh, de = _run(h, e, t, kind="alg_ce", n=8, c=2.)
    o2, t2, dh2, de2 = _oracle(h, e, t, "alg_ce", 8, 2.)
    np.testing.assert_allclose(obj.item(), o2.item(), rtol=.002, atol=.0002)
    np.testing.assert_allclose(tel.double(), t2, rtol=.02, atol=2e-7)
    assert rel_l2(dh, dh2) < .01
    assert rel_l2(de, de2) < .01


@pytest.mark.parametrize("ignore", [None, -100])
@pytest.mark.parametrize("V", [5000, 50304])
def test_ce_head_with_padded_vocab_and_ignore_index(ignore, V):
    """ce head at the benchmark shapes: loss within 1e-4 absolute, labels bit-exact.

    With ignore=None a -100 label matches no column, as the reference kernel's
    compare does; with ignore=-100 those rows leave the loss and the mean.
    """
    h, e, t = _inputs(512, 256, V, 0.02, 3, ignore_frac=0.05)
    obj, tel, dh, de = _run(h, e, t, kind="ce", ignore_index=ignore)
    o2, t2, dh2, de2 = _oracle(h, e, t, "ce", 16, 16., ignore_index=ignore)
    assert abs(obj.item() - o2.item()) < 1e-4
    np.testing.assert_allclose(tel.double(), t2, atol=2e-4, rtol=1e-4)
    if ignore is not None:
        assert torch.all(tel[t == -100] == 0)
    assert rel_l2(dh, dh2) < 1e-2
    assert rel_l2(de, de2) < 1e-2


@pytest.mark.parametrize("V", [5000, 50304])
def test_alg_ce_head_with_ignore_index(V):
    """alg_ce n=8 c=2 (the algebraic preset's head) with 5% of labels =
    ignore_index: most warps of the dz epilogue then hold an ignored row next
    to valid ones; ignored rows leave the objective and get exactly zero dh and
    telemetry; objective and gradients against the float64 oracle."""
    h, e, t = _inputs(512, 256, V, 0.02, 5, ignore_frac=0.05)
    obj, tel, dh, de = _run(h, e, t, kind="alg_ce", n=8, c=2., ignore_index=-100)
    o2, t2, dh2, de2 = _oracle(h, e, t, "alg_ce", 8, 2., ignore_index=-100)
    np.testing.assert_allclose(obj.item(), o2.item(), rtol=2e-3, atol=2e-4)
    np.testing.assert_allclose(tel.double(), t2, rtol=2e-2, atol=2e-4)
    ign = t == -100
    assert int(ign.sum()) > 0
    assert torch.all(tel[ign] == 0) and torch.all(dh[ign] == 0)
    assert rel_l2(dh, dh2) < 1e-2
    assert rel_l2(de, de2) < 1e-2


@pytest.mark.parametrize("key,kind,n,c", [("head_alg_n8c2", "alg_ce", 8, 2.0),
                                          ("head_alg_n16c16", "alg_ce", 16, 16.0), ("head_ce", "ce", 16, 16.0)])
def test_head_against_reference_goldens(key, kind, n, c):
    """Kernel vs outputs of the reference's dense head (tests/golden), bf16 I/O."""
    h, e, t = cases.head_inputs(31)
    obj, tel, dh, de = _run(torch.from_numpy(h).to(torch.bfloat16), torch.from_numpy(e), torch.from_numpy(t),
                            kind=kind, n=n, c=c)
    g = f"{key}_bf16"
    np.testing.assert_allclose(obj.item(), GOLD[g + "_obj"], rtol=2e-3, atol=2e-4)
    assert rel_l2(tel, torch.from_numpy(GOLD[g + "_tel"])) < 2e-2
    assert rel_l2(dh, torch.from_numpy(GOLD[g + "_dh"])) < 2e-2
    assert rel_l2(de, torch.from_numpy(GOLD[g + "_de"])) < 2e-2


def test_baseline_config3_full_size_against_chunked_check():
    """N=16384, d=768, V=50304 ce with 5% ignore_index=-100: objective within 1e-4 of a
    chunked float32 evaluation of the same formula on the GPU; dh, dE rel-L2 < 1e-2."""
    N, d, V = 16384, 768, 50304
    g = torch.Generator(device="cuda").manual_seed(11)
    h = torch.randn((N, d), device="cuda", generator=g).to(torch.bfloat16)
    e = (torch.randn((V, d), device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    t = torch.randint(0, V, (N,), device="cuda", generator=g)
    t[torch.rand(N, device="cuda", generator=g) < 0.05] = -100
    hc, ec = h.clone().requires_grad_(True), e.clone().requires_grad_(True)
    obj, tel = fused_head(hc, ec, t, kind="ce", ignore_index=-100)
    obj.backward()
    valid = t != -100
    cnt = int(valid.sum())
    ef = e.float()
    lse = torch.empty(N, device="cuda")
    ztt = torch.zeros(N, device="cuda")
    dh_ref = torch.zeros((N, d), device="cuda")
    de_ref = torch.zeros((V, d), device="cuda")
    for s in range(0, N, 1024):
        z = h[s:s + 1024].float() @ ef.T
        lse[s:s + 1024] = torch.logsumexp(z, -1)
        tt = t[s:s + 1024]
        ok = tt >= 0
        ztt[s:s + 1024][ok] = z[ok.nonzero()[:, 0], tt[ok]]
        p = torch.exp(z - lse[s:s + 1024, None])
        p[ok.nonzero()[:, 0], tt[ok]] -= 1
        p[~valid[s:s + 1024]] = 0
        dz = (p / cnt).to(torch.bfloat16).float()
        dh_ref[s:s + 1024] = dz @ ef
        de_ref += dz.T @ h[s:s + 1024].float()
    loss_ref = float(((lse - ztt)[valid]).sum() / cnt)
    assert abs(obj.item() - loss_ref) < 1e-4
    assert rel_l2(hc.grad.float(), dh_ref) < 1e-2
    assert rel_l2(ec.grad.float(), de_ref) < 1e-2


def test_out_of_range_label_sets_the_device_error_word():
    """With ignore_index set, a label outside [0, V) other than ignore_index is an
    error (the reference's kernel reads nothing for it, fused_head.py:86-87): the
    head sets DEV_ERR_BAD_LABEL (4) in the device error word, which
    algx_device_error() reads and clears; a following call with valid labels
    leaves the word at 0. Host-visible status only, no fault."""
    from algx import _lib as L
    V = 1000
    h, e, t = _inputs(256, 128, V, 0.05, 17)
    t[3] = -100          # the ignore index: fine
    L.device_error()     # start from a clear word
    for bad in (V, -1, 2 ** 31 - 1):
        tb = t.clone()
        tb[7] = bad
        _run(h, e, tb, kind="ce", ignore_index=-100)
        assert L.device_error() == 4, bad
        assert L.device_error() == 0  # read-and-clear
    _run(h, e, t, kind="ce", ignore_index=-100)
    assert L.device_error() == 0
