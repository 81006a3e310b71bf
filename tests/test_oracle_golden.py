"""Pin the CPU oracle against outputs of the reference's own dense code.

``tests/golden/reference_dense.npz`` was produced by running the reference's
``algebraic.py`` / ``standard.py`` / ``evaluation.py`` source (see
``tests/golden/make_golden.py``). Inputs are regenerated from seeds; a
checksum guards against generator drift.
"""

import numpy as np
import pytest
import torch

from oracle import reference_math as R
from tests.golden import cases

GOLD = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__),
                                          "golden", "reference_dense.npz"))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def test_fixture_inputs_regenerate():
    for idx, (name, n, c, with_sink, scale) in enumerate(cases.ATTN_CASES):
        q, k, v, g, _ = cases.attn_inputs(100 + 10 * idx, scale=scale, with_sink=with_sink)
        s = sum(float(np.sum(a, dtype=np.float64)) for a in (q, k, v, g))
        assert s == float(GOLD[f"attn_{name}_checksum"])
    x, gain, dy = cases.norm_inputs(7)
    assert sum(float(np.sum(a, dtype=np.float64)) for a in (x, gain, dy)) == float(GOLD["norm_checksum"])


@pytest.mark.parametrize("case", cases.ATTN_CASES, ids=[c[0] for c in cases.ATTN_CASES])
@pytest.mark.parametrize("prec", ["f64", "bf16"])
def test_attention_oracle_matches_reference(case, prec):
    name, n, c, with_sink, scale = case
    idx = cases.ATTN_CASES.index(case)
    q, k, v, g, sink = cases.attn_inputs(100 + 10 * idx, scale=scale, with_sink=with_sink)
    io = torch.bfloat16 if prec == "bf16" else None
    qt, kt, vt = (cases.to_io(a, io) for a in (q, k, v))
    gt = torch.from_numpy(g).double()
    st = None if sink is None else torch.from_numpy(sink).double()

    def dense(q_, k_, v_, s_):
        return R.asinh_attention(q_, k_, v_, n=n, c=c, sink_logit=s_, io_dtype=io)

    o, dq, dk, dv, ds = R.attention_grads(dense, qt, kt, vt, gt, st)
    key = f"attn_{name}_{prec}"
    tol_o, tol_g = (2e-6, 2e-6) if prec == "f64" else (8e-3, 2e-2)
    assert rel_l2(o, GOLD[key + "_o"]) < tol_o
    for nm, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert rel_l2(t, GOLD[key + "_" + nm]) < tol_g, nm
    if with_sink:
        assert rel_l2(ds, GOLD[key + "_dsink"]) < tol_g

    # The kernel-level function (scale fold, guarded/shifted/clipped variants)
    # equals the dense one wherever the clamp does not bind.
    if prec == "f64":
        for opts in (dict(range_guard=True), dict(shift=True), dict(shift=False)):
            def flash(q_, k_, v_, s_):
                return R.flash_attention(q_, k_, v_, s_, kind="asinh", n=n, c=c, **opts)
            o2, dq2, dk2, dv2, ds2 = R.attention_grads(flash, qt, kt, vt, gt, st)
            assert rel_l2(o2, o) < 1e-12
            for a, b in ((dq2, dq), (dk2, dk), (dv2, dv)):
                assert rel_l2(a, b) < 1e-10
            if with_sink:
                assert rel_l2(ds2, ds) < 1e-10


@pytest.mark.parametrize("eps", [1e-5, 1e-3])
@pytest.mark.parametrize("prec", ["f64", "bf16"])
def test_rms_norm_oracle_matches_reference(eps, prec):
    x, gain, dy = cases.norm_inputs(7)
    io = torch.bfloat16 if prec == "bf16" else None
    xt = cases.to_io(x, io)
    gt = torch.from_numpy(gain).double()
    dyt = torch.from_numpy(dy).double()
    y = R.rms_norm(xt, gt, eps, io_dtype=io)
    dx, dg = R.qk_norm_backward(xt, gt, dyt, eps)
    key = f"norm_eps{eps:g}_{prec}"
    if prec == "f64":
        assert rel_l2(y, GOLD[key + "_y"]) < 1e-7
        assert rel_l2(dx, GOLD[key + "_dx"]) < 1e-7
        assert rel_l2(dg, GOLD[key + "_dgain"]) < 1e-7
    else:
        assert rel_l2(y, GOLD[key + "_y"]) < 4e-3
        assert rel_l2(dx, GOLD[key + "_dx"]) < 1e-2
        assert rel_l2(dg, GOLD[key + "_dgain"]) < 1e-2


@pytest.mark.parametrize("n,c", [(16, 16.0), (8, 2.0)])
def test_likelihood_oracle_matches_reference(n, c):
    z = torch.from_numpy(cases.normal(21, (7, 300), 6.0)).double()
    t = torch.tensor([0, 5, 299, 17, 17, 100, -100])
    key = f"lik_n{n}c{c:g}"
    obj, pt = R.algebraic_likelihood(z, t, n, c)
    np.testing.assert_allclose(obj.item(), GOLD[key + "_obj"], rtol=1e-12)
    np.testing.assert_allclose(pt.numpy(), GOLD[key + "_pt"], rtol=1e-10)
    grad = R.algebraic_likelihood_grad(z, t, n, c)
    np.testing.assert_allclose(grad.numpy(), GOLD[key + "_grad"], rtol=1e-9, atol=1e-15)
    obj_l, pt_l = R.algebraic_likelihood_lean(z, t, n, c)
    np.testing.assert_allclose(obj_l.item(), GOLD[key + "_lean_obj"], rtol=1e-12)
    np.testing.assert_allclose(pt_l.numpy(), GOLD[key + "_lean_pt"], rtol=1e-10)
    np.testing.assert_allclose(R.logprob_from_logits(z, t, "alg_ce", n, c).numpy(),
                               GOLD[key + "_logprob"], rtol=1e-10)


def test_cross_entropy_oracle_matches_reference():
    z = torch.from_numpy(cases.normal(21, (7, 300), 6.0)).double().requires_grad_(True)
    t = torch.tensor([0, 5, 299, 17, 17, 100, -100])
    obj, nll = R.cross_entropy(z, t)
    obj.backward()
    # standard.py:43 casts the logits to float32, so the reference value
    # carries float32 rounding; the oracle stays float64.
    np.testing.assert_allclose(obj.item(), GOLD["ce_obj"], rtol=2e-7)
    np.testing.assert_allclose(nll.numpy(), GOLD["ce_nll"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(z.grad.numpy(), GOLD["ce_grad"], rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("kind,n,c", [("alg_ce", 8, 2.0), ("alg_ce", 16, 16.0), ("ce", 0, 0.0)])
@pytest.mark.parametrize("prec", ["f64", "bf16"])
def test_fused_head_oracle_matches_reference(kind, n, c, prec):
    """The fused kernel's function (additive rho^n, clamp, root stat) = the dense head."""
    h, e, t = cases.head_inputs(31)
    io = torch.bfloat16 if prec == "bf16" else None
    ht = cases.to_io(h, io)
    et = torch.from_numpy(e).double()
    tt = torch.from_numpy(t)
    key = f"head_ce_{prec}" if kind == "ce" else f"head_alg_n{n}c{c:g}_{prec}"
    obj, tel, _, _ = R.fused_head_forward(ht, et, tt, kind=kind, n=n, c=c, io_dtype=io)
    dh, de = R.fused_head_backward(ht, et, tt, kind=kind, n=n, c=c, io_dtype=io)
    if prec == "f64":
        np.testing.assert_allclose(obj.item(), GOLD[key + "_obj"], rtol=1e-6)
        assert rel_l2(tel, GOLD[key + "_tel"]) < 1e-6
        assert rel_l2(dh, GOLD[key + "_dh"]) < 1e-6
        assert rel_l2(de, GOLD[key + "_de"]) < 1e-6
    else:
        np.testing.assert_allclose(obj.item(), GOLD[key + "_obj"], rtol=2e-3, atol=2e-4)
        assert rel_l2(tel, GOLD[key + "_tel"]) < 2e-2
        assert rel_l2(dh, GOLD[key + "_dh"]) < 1e-2
        assert rel_l2(de, GOLD[key + "_de"]) < 1e-2


ALU = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "reference_alu.npz"))


def _alu_inputs():
    x = cases.normal(41, (6, 256), 4.0)
    x[0, :8] = np.array([0.0, -1e-3, 1e-3, -30.0, 30.0, -300.0, 300.0, -3000.0], dtype=np.float32)
    return x, cases.normal(42, (6, 256))


@pytest.mark.parametrize("beta", [0.5, 1.0])
@pytest.mark.parametrize("prec", ["f64", "bf16"])
def test_alu_oracle_matches_reference(beta, prec):
    """ALU-GLU's activation and its custom VJP (algebraic.py:86-113) against the reference's own code."""
    x, g = _alu_inputs()
    assert float(np.sum(x, dtype=np.float64)) + float(np.sum(g, dtype=np.float64)) == float(ALU["alu_checksum"])
    io = torch.bfloat16 if prec == "bf16" else None
    xt = cases.to_io(x, io if io else torch.float64).requires_grad_(True)
    y = R.alu(xt, beta, io_dtype=io)
    y.backward(cases.to_io(g, io if io else torch.float64))
    key = f"alu_b{beta:g}_{prec}"
    tol = 1e-6 if prec == "f64" else 1e-2
    assert rel_l2(y.detach().numpy(), ALU[key + "_y"]) < tol
    assert rel_l2(xt.grad.numpy(), ALU[key + "_dx"]) < tol
    # the far negative tail keeps its precision (r^2 / (1 - u) branch)
    assert np.all(np.isfinite(ALU[key + "_y"]))
