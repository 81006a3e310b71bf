"""The reference's own optimizer test cases (tests/test_optimizers.py:28-298),
restated on torch tensors against algx.optim with the reference's shapes,
tolerances and call sequences. The random matrices are torch draws (JAX's
PRNGKey streams are not reproducible here); the bounds are structural, so
they hold for any standard-normal draw. The two jax.jit cases
(test_optimizers.py:167-181, 284-298) have no counterpart: the update is
plain torch code."""

import torch

from algx import optim as O


def _normal(seed, *shape):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed))


# ---------------------------------------------- Newton-Schulz (:28-91)
def test_newton_schulz_square_matrix():
    o32 = O.newton_schulz_5(_normal(42, 32, 32), steps=5)
    assert float(torch.linalg.norm(o32 @ o32.T - torch.eye(32))) < 1.0
    o64 = O.newton_schulz_5(_normal(101, 64, 64), steps=5)
    assert float((o64 @ o64.T - torch.eye(64)).abs().max()) < 0.25


def test_newton_schulz_tall_matrix():
    o = O.newton_schulz_5(_normal(102, 128, 64), steps=5)
    assert o.shape == (128, 64)
    assert float((o.T @ o - torch.eye(64) * (128.0 / 64.0)).abs().max()) < 1.0


def test_newton_schulz_wide_matrix():
    o = O.newton_schulz_5(_normal(103, 64, 128), steps=5)
    assert o.shape == (64, 128)
    assert float((o @ o.T - torch.eye(64)).abs().max()) < 0.25


def test_newton_schulz_batched_3d():
    o = O.newton_schulz_5(_normal(104, 4, 32, 32), steps=5)
    assert o.shape == (4, 32, 32)
    assert float((o @ o.transpose(-2, -1) - torch.eye(32)).abs().max()) < 0.25


def test_newton_schulz_zero_norm_guard():
    o = O.newton_schulz_5(torch.zeros(16, 16), steps=5)
    assert torch.isfinite(o).all() and torch.allclose(o, torch.zeros(16, 16))


def test_newton_schulz_singular_value_bound():
    sv = torch.linalg.svdvals(O.newton_schulz_5(_normal(777, 32, 32), steps=5))
    assert float((sv - 1.0).abs().max()) < 0.15


# ------------------------------------------------ routing (:94-118)
def test_muon_param_internal_matrices():
    for key in ["w_q", "w_k", "w_v", "w_o", "w_g", "w_u", "w_d"]:
        assert O.is_muon_param(("layers", key), torch.zeros(12, 64, 64)) is True, key


def test_non_muon_params_vector_and_embedding():
    non_muon = [(("embed",), torch.zeros(32768, 768)), (("embed_gain",), torch.zeros(768)),
                (("final_gain",), torch.zeros(768)), (("layers", "ln1"), torch.zeros(12, 768)),
                (("layers", "ln2"), torch.zeros(12, 768)), (("layers", "q_gain"), torch.zeros(12, 64)),
                (("layers", "k_gain"), torch.zeros(12, 64)), (("layers", "sink"), torch.zeros(12, 12))]
    for path, param in non_muon:
        assert O.is_muon_param(path, param) is False, path


# ---------------------------------------------- muon_adamw (:121-164)
def test_muon_adamw_registration_and_types():
    init_fn, step_fn = O.get_optimizer("muon_adamw", lr=0.003, total_steps=100)
    assert callable(init_fn) and callable(step_fn)
    state = init_fn({"w_q": torch.ones(16, 16), "embed_gain": torch.ones(16)})
    assert isinstance(state, O.OptState)
    assert int(state.count) == 0
    assert "w_q" in state.m
    assert state.v.get("w_q") is None and state.v.get("embed_gain") is not None


def test_muon_nesterov_momentum_update():
    init_fn, step_fn = O.get_optimizer("muon_adamw", lr=0.01, muon_momentum=0.95, total_steps=10)
    params = {"w_q": torch.ones(16, 16)}
    new_params, new_state = step_fn(0, params, {"w_q": torch.ones(16, 16) * 0.1}, init_fn(params), {"w_q": True})
    assert not torch.allclose(new_params["w_q"], params["w_q"])
    assert int(new_state.count) == 1
    assert not torch.allclose(new_state.m["w_q"], torch.zeros(16, 16))


def test_muon_adamw_cosine_schedule():
    init_fn, step_fn = O.get_optimizer("muon_adamw", lr=0.01, total_steps=100, warmup_fraction=0.02,
                                       min_lr_ratio=0.1)
    params = {"embed_gain": torch.ones(16)}
    state = init_fn(params)
    grads = {"embed_gain": torch.ones(16) * 0.1}
    p0, _ = step_fn(0, params, grads, state, {"embed_gain": False})
    p50, _ = step_fn(50, params, grads, state, {"embed_gain": False})
    assert not torch.allclose(params["embed_gain"] - p0["embed_gain"], params["embed_gain"] - p50["embed_gain"])


# --------------------------------------------------- cadamw (:184-245)
def test_cadamw_registration():
    init_fn, step_fn = O.get_optimizer("cadamw", lr=0.003, total_steps=100)
    assert callable(init_fn) and callable(step_fn)
    assert init_fn({"w": torch.ones(4, 4)}).v.get("w") is not None


def test_cadamw_descent_monotonicity():
    init_fn, step_fn = O.get_optimizer("cadamw", lr=0.01, total_steps=10)
    p = {"w": torch.ones(8)}
    g = {"w": torch.tensor([1.0, -1.0, 0.5, -0.5, 2.0, -2.0, 0.1, -0.1])}
    p1, _ = step_fn(0, p, g, init_fn(p), {"w": False})
    assert ((p["w"] - p1["w"]) * g["w"] >= -1e-6).all()


def test_cadamw_cautious_mask_opposition():
    init_fn, step_fn = O.get_optimizer("cadamw", lr=0.01, total_steps=100)
    p = {"x": torch.zeros(4)}
    p1, s1 = step_fn(0, p, {"x": torch.tensor([1.0, 1.0, 1.0, 1.0])}, init_fn(p), {"x": False})
    p2, _ = step_fn(1, p1, {"x": torch.tensor([-1.0, 1.0, 1.0, 1.0])}, s1, {"x": False})
    assert torch.isfinite(p2["x"]).all()


def test_cadamw_decoupled_weight_decay():
    init_fn, step_fn = O.get_optimizer("cadamw", lr=0.01, weight_decay=0.1, total_steps=100)
    p = {"w_decay": torch.ones(8), "w_nodecay": torch.ones(8)}
    g = {"w_decay": torch.zeros(8), "w_nodecay": torch.zeros(8)}
    p1, _ = step_fn(0, p, g, init_fn(p), {"w_decay": True, "w_nodecay": False})
    assert float(p1["w_decay"][0]) < 1.0
    assert torch.isclose(p1["w_nodecay"][0], torch.tensor(1.0))


def test_cadamw_zero_gradient_step():
    init_fn, step_fn = O.get_optimizer("cadamw", lr=0.01, total_steps=100)
    p = {"x": torch.ones(8)}
    p1, _ = step_fn(0, p, {"x": torch.zeros(8)}, init_fn(p), {"x": False})
    assert torch.allclose(p1["x"], p["x"])


def test_cadamw_scalar_parameter():
    init_fn, step_fn = O.get_optimizer("cadamw", lr=0.01, total_steps=100)
    p = {"scalar": torch.tensor(2.0)}
    p1, _ = step_fn(0, p, {"scalar": torch.tensor(0.5)}, init_fn(p), {"scalar": False})
    assert p1["scalar"].shape == () and torch.isfinite(p1["scalar"]).all()


# ---------------------------------------- hybrid_muon_cadamw (:248-282)
def test_hybrid_registration_and_state():
    init_fn, step_fn = O.get_optimizer("hybrid_muon_cadamw", lr=0.003, total_steps=100)
    assert callable(init_fn) and callable(step_fn)
    state = init_fn({"embed": torch.zeros(32, 16), "w_q": torch.zeros(16, 16)})
    assert hasattr(state, "count") and hasattr(state, "m") and hasattr(state, "v")
    assert state.v.get("w_q") is None and state.v.get("embed") is not None


def test_hybrid_step_joint_execution():
    init_fn, step_fn = O.get_optimizer("hybrid_muon_cadamw", lr=0.01, total_steps=100)
    params = {"w_q": torch.ones(16, 16), "embed_gain": torch.ones(16)}
    grads = {"w_q": torch.ones(16, 16) * 0.05, "embed_gain": torch.ones(16) * 0.05}
    new_params, _ = step_fn(0, params, grads, init_fn(params), {"w_q": True, "embed_gain": False})
    for k in params:
        assert torch.isfinite(new_params[k]).all()
        assert not torch.allclose(new_params[k], params[k])


def test_hybrid_empty_pytree():
    init_fn, step_fn = O.get_optimizer("hybrid_muon_cadamw", lr=0.01, total_steps=10)
    p1, _ = step_fn(0, {}, {}, init_fn({}), {})
    assert p1 == {}
