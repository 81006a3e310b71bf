"""algx.optim against outputs of the reference's own optimizers.py
(tests/golden/reference_optim.npz, made by tests/golden/make_golden.py from
the reference's unchanged source on the torch stand-in for JAX): the
Newton-Schulz orthogonalisation, the cosine schedule, and three steps of
muon_adamw, cadamw and hybrid_muon_cadamw on a parameter tree with every
routing class, all float64, through both interfaces: the reference's own
get_optimizer / init_fn / step_fn, and the in-place ReferenceOptimizer."""

import os

import numpy as np
import pytest
import torch

from algx import optim as O
from tests.golden import cases

GOLD = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_optim.npz"))


@pytest.mark.parametrize("shape", cases.OPTIM_NS_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_newton_schulz_matches_reference(shape):
    key = "ns5_" + "x".join(map(str, shape))
    g = torch.from_numpy(cases.normal(61 + cases.OPTIM_NS_SHAPES.index(shape), shape)).double()
    assert np.array_equal(g.numpy(), GOLD[key + "_in"])  # the fixture's input is regenerated exactly
    np.testing.assert_allclose(O.newton_schulz_5(g).numpy(), GOLD[key], rtol=1e-10, atol=1e-12)


def test_newton_schulz_output_is_nearly_orthogonal():
    g = torch.from_numpy(cases.normal(5, (32, 64))).double()
    x = O.newton_schulz_5(g)
    sv = torch.linalg.svdvals(x)
    assert float(sv.max()) < 1.2 and float(sv.min()) > 0.5  # quintic NS lands near 1, not exactly


def test_cosine_schedule_matches_reference():
    lr = O.cosine_schedule(2e-2, 10, 0.2, 0.1)
    got = np.array([float(lr(t)) for t in range(13)])
    np.testing.assert_array_equal(got, GOLD["schedule"])


def test_routing_follows_the_reference_rule():
    assert O.is_muon_param("layers.3.w_qkv", 2) and O.is_muon_param("w_d", 2)
    assert not O.is_muon_param("embed", 2)
    for n in ("layers.0.ln1", "layers.0.q_gain", "final_gain", "layers.0.sink", "bias"):
        assert not O.is_muon_param(n, 1)


@pytest.mark.parametrize("name", O.NAMES)
def test_three_steps_match_reference(name):
    params0, grads = cases.optim_inputs(71)
    params = {k: torch.from_numpy(v).double() for k, v in params0.items()}
    for p in params.values():
        p.grad = torch.zeros_like(p)
    opt = O.ReferenceOptimizer(name, [(k, params[k], cases.OPTIM_DECAY[k]) for k in sorted(params)],
                               **cases.OPTIM_ARGS)
    for step, gr in enumerate(grads):
        for k, p in params.items():
            p.grad.copy_(torch.from_numpy(gr[k]).double())
        opt.step(step)
        for k, p in params.items():
            np.testing.assert_allclose(p.numpy(), GOLD[f"opt_{name}_step{step}_{k}"], rtol=1e-9, atol=1e-12,
                                       err_msg=f"{name} step {step} {k}")


@pytest.mark.parametrize("name", O.NAMES)
def test_fused_weights_update_like_separate_reference_matrices(name):
    """w_qkv = [w_q | w_k | w_v] and w_gu = [w_g | w_u] (column blocks) update
    exactly as the reference's separate matrices do."""
    g = torch.Generator().manual_seed(3)
    d, f = 8, 12
    mats = {k: torch.randn(d, f if k in ("w_g", "w_u") else d, generator=g, dtype=torch.float64)
            for k in ("w_q", "w_k", "w_v", "w_g", "w_u")}
    grads = [{k: 0.1 * torch.randn(v.shape, generator=g, dtype=torch.float64) for k, v in mats.items()}
             for _ in range(2)]
    sep = {k: v.clone() for k, v in mats.items()}
    for p in sep.values():
        p.grad = torch.zeros_like(p)
    fused = {"l.w_qkv": torch.cat([mats[k] for k in ("w_q", "w_k", "w_v")], 1).contiguous(),
             "l.w_gu": torch.cat([mats[k] for k in ("w_g", "w_u")], 1).contiguous()}
    for p in fused.values():
        p.grad = torch.zeros_like(p)
    o1 = O.ReferenceOptimizer(name, [(k, v, True) for k, v in sep.items()], lr=1e-2, total_steps=5)
    o2 = O.ReferenceOptimizer(name, [(k, v, True) for k, v in fused.items()], lr=1e-2, total_steps=5)
    for step, gr in enumerate(grads):
        for k, p in sep.items():
            p.grad.copy_(gr[k])
        fused["l.w_qkv"].grad.copy_(torch.cat([gr[k] for k in ("w_q", "w_k", "w_v")], 1))
        fused["l.w_gu"].grad.copy_(torch.cat([gr[k] for k in ("w_g", "w_u")], 1))
        o1.step(step)
        o2.step(step)
    assert torch.equal(fused["l.w_qkv"], torch.cat([sep[k] for k in ("w_q", "w_k", "w_v")], 1))
    assert torch.equal(fused["l.w_gu"], torch.cat([sep[k] for k in ("w_g", "w_u")], 1))


def test_batched_newton_schulz_equals_one_matrix_at_a_time():
    g = torch.from_numpy(cases.normal(9, (5, 12, 20))).double()
    batched = O.newton_schulz_5(g)
    for i in range(5):
        np.testing.assert_allclose(batched[i].numpy(), O.newton_schulz_5(g[i]).numpy(), rtol=1e-12, atol=1e-14)
    tall = g.transpose(-2, -1)  # the M > N branch, batched: transposed, then scaled by sqrt(M / N)
    np.testing.assert_allclose(O.newton_schulz_5(tall).numpy(), (batched.transpose(-2, -1) * (20 / 12) ** 0.5).numpy(),
                               rtol=1e-12, atol=1e-14)


def test_default_precision_rounds_the_operands_to_bf16():
    """precision="default": every matmul operand rounded to bf16 (XLA's DEFAULT
    f32 dot on TPU). Its result stays within bf16-level error of the exact
    orthogonalisation and is not the exact one."""
    g = torch.from_numpy(cases.normal(10, (3, 32, 48))).double()
    hi = O.newton_schulz_5(g, precision="highest")
    lo = O.newton_schulz_5(g, precision="default")
    rel = float(torch.linalg.norm(lo - hi) / torch.linalg.norm(hi))
    assert 1e-5 < rel < 3e-2, rel
    sv = torch.linalg.svdvals(lo)
    assert float(sv.max()) < 1.2 and float(sv.min()) > 0.5


def test_unknown_precision_is_rejected():
    with pytest.raises(ValueError, match="precision"):
        O.ReferenceOptimizer("muon_adamw", [], lr=1e-3, precision="bf16")
    with pytest.raises(ValueError, match="precision"):
        O.newton_schulz_5(torch.zeros(4, 4), precision="high")


@pytest.mark.parametrize("name", O.NAMES)
def test_get_optimizer_matches_reference(name):
    """The reference's own call sequence (get_optimizer, init_fn, step_fn per
    step with a decay mask, as tests/golden/make_golden.py drives the
    reference) reproduces its parameters step by step; the inputs are not
    modified and Muon-routed leaves hold no second moment."""
    params0, grads = cases.optim_inputs(71)
    mask = {k: torch.tensor(v) for k, v in cases.OPTIM_DECAY.items()}
    init_fn, step_fn = O.get_optimizer(name, **cases.OPTIM_ARGS)
    first = {k: torch.from_numpy(v).double() for k, v in params0.items()}
    params = first
    state = init_fn(params)
    for step, gr in enumerate(grads):
        params, state = step_fn(step, params, {k: torch.from_numpy(v).double() for k, v in gr.items()}, state, mask)
        for k, p in params.items():
            np.testing.assert_allclose(p.numpy(), GOLD[f"opt_{name}_step{step}_{k}"], rtol=1e-9, atol=1e-12,
                                       err_msg=f"{name} step {step} {k}")
    assert int(state.count) == len(grads)
    for k, v in params0.items():
        assert np.array_equal(first[k].numpy(), v)
    for k in params0:
        muon = name != "cadamw" and O.is_muon_param(k, params0[k].ndim)
        assert (state.v[k] is None) == muon


def test_get_optimizer_walks_nested_trees_and_fused_leaves():
    """Nested dicts and lists, the reference model's layout, update as flat
    leaves; a fused w_qkv leaf updates as its three reference matrices."""
    g = torch.Generator().manual_seed(8)
    mk = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    sep = {"layers": [{"w_q": mk(8, 8), "w_k": mk(8, 8), "w_v": mk(8, 8), "ln1": mk(8)} for _ in range(2)],
           "embed": mk(10, 8)}
    fused = {"layers": [{"w_qkv": torch.cat([l["w_q"], l["w_k"], l["w_v"]], 1), "ln1": l["ln1"].clone()}
                        for l in sep["layers"]], "embed": sep["embed"].clone()}
    gs = {"layers": [{"w_q": mk(8, 8), "w_k": mk(8, 8), "w_v": mk(8, 8), "ln1": mk(8)} for _ in range(2)],
          "embed": mk(10, 8)}
    gf = {"layers": [{"w_qkv": torch.cat([l["w_q"], l["w_k"], l["w_v"]], 1), "ln1": l["ln1"]} for l in gs["layers"]],
          "embed": gs["embed"]}
    dm_s = {"layers": [{"w_q": True, "w_k": True, "w_v": True, "ln1": False}] * 2, "embed": True}
    dm_f = {"layers": [{"w_qkv": True, "ln1": False}] * 2, "embed": True}
    init_fn, step_fn = O.get_optimizer("hybrid_muon_cadamw", lr=1e-2, total_steps=5)
    ps, st_s = step_fn(0, sep, gs, init_fn(sep), dm_s)
    pf, st_f = step_fn(0, fused, gf, init_fn(fused), dm_f)
    for i in range(2):
        assert torch.equal(pf["layers"][i]["w_qkv"],
                           torch.cat([ps["layers"][i][k] for k in ("w_q", "w_k", "w_v")], 1))
        assert torch.equal(pf["layers"][i]["ln1"], ps["layers"][i]["ln1"])
        assert st_f.v["layers"][i]["w_qkv"] is None and st_f.v["layers"][i]["ln1"] is not None
    assert torch.equal(pf["embed"], ps["embed"])


def test_unknown_optimizer_name_is_rejected():
    with pytest.raises(ValueError, match="Unknown optimizer"):
        O.ReferenceOptimizer("sgd", [], lr=1e-3)
    with pytest.raises(ValueError, match="Unknown optimizer: sgd"):
        O.get_optimizer("sgd", lr=1e-3)
