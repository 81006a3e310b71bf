"""Known-answer identities of the reference (tests/test_components.py:18-108), on the oracle."""

import numpy as np
import pytest
import torch

from oracle import reference_math as R


def test_rho_identities():
    x = torch.linspace(-50, 50, 1001, dtype=torch.float64)
    y = torch.linspace(-3, 7, 1001, dtype=torch.float64)
    np.testing.assert_allclose(R.rho(x), np.exp(np.arcsinh(x.numpy())), rtol=1e-12)
    np.testing.assert_allclose(R.rho(x) * R.rho(-x), 1.0, rtol=1e-12)
    oplus = x * torch.sqrt(1 + y * y) + y * torch.sqrt(1 + x * x)
    np.testing.assert_allclose(R.rho(x) * R.rho(y), R.rho(oplus), rtol=1e-10)


@pytest.mark.parametrize("n,c", [(8, 1.0), (16, 16.0), (32, 4.0)])
def test_asinh_weights_equal_softmax_of_compressed_logits(n, c):
    g = torch.Generator().manual_seed(0)
    s = torch.randn((2, 3, 7, 7), generator=g, dtype=torch.float64) * 5
    mask = torch.tril(torch.ones((7, 7), dtype=torch.bool))[None, None]
    b = torch.full((1, 3, 1, 1), 0.7, dtype=torch.float64)
    w = R.asinh_power_weights(s, mask, n, c, b)
    logits = torch.where(mask, n * torch.asinh(s / c), torch.full_like(s, -float("inf")))
    full = torch.cat([logits, torch.broadcast_to(n * torch.asinh(b / c), s.shape[:-1] + (1,))], -1)
    ref = torch.softmax(full, -1)[..., :-1]
    np.testing.assert_allclose(w, ref, rtol=1e-10, atol=1e-14)
    big = R.asinh_power_weights(s * 1e6, mask, n, c, None)
    assert torch.isfinite(big).all() and torch.allclose(big.sum(-1), torch.ones(()).double())


@pytest.mark.parametrize("n,c", [(16, 16.0), (8, 2.0)])
def test_algebraic_likelihood_gradient_is_exact_log_loss_gradient(n, c):
    g = torch.Generator().manual_seed(1)
    z = (torch.randn((6, 11), generator=g, dtype=torch.float64) * 4).requires_grad_(True)
    t = torch.tensor([0, 3, 10, 5, 5, 1])
    true_nll = -torch.mean(R.logprob_from_logits(z, t, "alg_ce", n, c))
    true_nll.backward()
    grad = R.algebraic_likelihood_grad(z.detach(), t, n, c)
    np.testing.assert_allclose(grad, z.grad, rtol=1e-9, atol=1e-12)
    pt = R.algebraic_likelihood(z.detach(), t, n, c)[1]
    np.testing.assert_allclose(np.log(pt.numpy()),
                               R.logprob_from_logits(z.detach(), t, "alg_ce", n, c), rtol=1e-9)


@pytest.mark.parametrize("n,c", [(16, 16.0), (8, 2.0)])
def test_lean_likelihood_equals_exact(n, c):
    g = torch.Generator().manual_seed(3)
    z = torch.randn((7, 300), generator=g, dtype=torch.float64) * 6
    t = torch.tensor([0, 5, 299, 17, 17, 100, 3])
    o1, p1 = R.algebraic_likelihood_lean(z, t, n, c)
    o2, p2 = R.algebraic_likelihood(z, t, n, c)
    np.testing.assert_allclose(p1, p2, rtol=1e-9)


def test_clamps_match_reference_constants():
    # make_variant: T=512 -> 69.51, T=2048 -> 63.75 (n=16); fused head V=50304
    assert abs(R.attention_clamp(512, 16) - 69.51) < 0.01
    assert abs(R.attention_clamp(2048, 16) - 63.75) < 0.01
    assert abs(R.likelihood_clamp(50304, 8) - 3632.8) < 0.1
    assert abs(R.likelihood_clamp(50304, 16) - 30.14) < 0.01


def test_clipped_vjp_is_zero_above_cap():
    """kernels/flash.py:357-360 and tests/test_flash_kernel_tpu.py:122-138 on the oracle."""
    shape = (1, 1, 32, 64)
    q = torch.full(shape, 1000 ** 0.5, dtype=torch.float64)
    v = torch.randn(shape, dtype=torch.float64, generator=torch.Generator().manual_seed(39))
    g = torch.randn(shape, dtype=torch.float64, generator=torch.Generator().manual_seed(40))
    sink = torch.full((1,), 1000.0, dtype=torch.float64)

    def fn(q_, k_, v_, s_):
        return R.flash_attention(q_, k_, v_, s_, kind="asinh", n=16, c=8.0, shift=False)

    _, dq, dk, _, ds = R.attention_grads(fn, q, q.clone(), v, g, sink)
    assert torch.all(dq == 0) and torch.all(dk == 0) and torch.all(ds == 0)


def test_cayley_powers_closed_form():
    """((1 + i w)^2 / (1 + w^2))^m = exp(2 i m atan w): the binary exponentiation of
    algebraic.py:124-149 (float64 here) against the closed form."""
    w = torch.tensor([0.5, 0.1, 0.003, 0.0], dtype=torch.float64)
    c, s = R.cayley_powers(w, 2048)
    ang = 2 * torch.arange(2048, dtype=torch.float64)[:, None] * torch.atan(w)[None, :]
    assert torch.allclose(c, torch.cos(ang), atol=1e-11) and torch.allclose(s, torch.sin(ang), atol=1e-11)


def test_rotary_is_a_rotation():
    """apply_rotary keeps row norms and its transpose undoes it (the VJP the fused epilogue applies)."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn((2, 3, 64, 64), generator=g, dtype=torch.float64)
    cos, sin = R.rope_table(64, 80, dtype=torch.float64)
    y = R.apply_rotary(x, cos, sin)
    assert torch.allclose(y.norm(dim=-1), x.norm(dim=-1), rtol=1e-12)
    back = R.apply_rotary(y, cos, -sin)
    assert torch.allclose(back, x, atol=1e-12)


def test_product_tables_match_oracle():
    """algx.rotary builds the same fp32 tables as the oracle's restatement."""
    from algx import rotary as P
    for got, want in ((P.rope_table(64, 2048), R.rope_table(64, 2048)),
                      (P.cayley_table_geometric(64, 2048), R.cayley_table_geometric(64, 2048)),
                      (P.cayley_table_geometric(64, 512, fraction=0.5), R.cayley_table_geometric(64, 512,
                                                                                                 fraction=0.5))):
        for a, b in zip(got, want):
            assert a.dtype == torch.float32 and a.shape == b.shape
            assert torch.allclose(a, b, atol=2e-6, rtol=0)


@pytest.mark.parametrize("beta", [0.5, 0.8, 1.0])
def test_alu_stable_form_and_custom_vjp_match_the_closed_form(beta):
    """alu(x) = x/2 (1 + bx / sqrt(1 + b^2 x^2)) (algebraic.py:95-101): the oracle's
    r^2 / (1 - u) branch for bx < 0 equals the direct formula where both are
    accurate, and its custom VJP (algebraic.py:104-113) equals autograd of it."""
    x = torch.linspace(-40.0, 40.0, 4001, dtype=torch.float64)
    xa = x.clone().requires_grad_(True)
    y = R.alu(xa, beta)
    y.sum().backward()
    xb = x.clone().requires_grad_(True)
    bz = beta * xb
    direct = 0.5 * xb * (1.0 + bz / torch.sqrt(1.0 + bz * bz))
    direct.sum().backward()
    torch.testing.assert_close(y.detach(), direct.detach(), rtol=1e-9, atol=1e-12)
    torch.testing.assert_close(xa.grad, xb.grad, rtol=1e-9, atol=1e-12)
    # far negative tail: the stable form keeps relative precision where 1 + u cancels
    # (for bx < 0, with w = 1/(bx)^2: 1 + u = w / ((1 + w) + sqrt(1 + w)), no cancellation)
    t = torch.tensor([-30.0, -1e4, -1e6], dtype=torch.float64)
    w = 1.0 / (beta * beta * t * t)
    exact = 0.5 * t * w / ((1.0 + w) + torch.sqrt(1.0 + w))
    torch.testing.assert_close(R.alu(t, beta), exact, rtol=1e-12, atol=0.0)
