"""GPU parity of the reference's pure algebraic preset pieces (config.py:25-36):
the ALU-GLU gate kernel against the oracle's ``alu`` (itself pinned to the
reference's own code by tests/test_oracle_golden.py), and the preset model
(ALU-GLU, geometric Cayley rotations, learned sink, ``alg_ce`` head) against a
float64 restatement of model.py.

Tolerances: ALU-GLU forward within one bf16 ulp of the oracle with the
reference's rounding points, backward within 1e-2 relative L2; the 2-layer
model's objective within 2e-3 relative and each parameter gradient within
3e-2 relative L2.
"""

import pytest
import torch

from oracle import reference_math as R

pytestmark = pytest.mark.gpu

F64 = torch.float64


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-300))


def _rb(x):
    return x + (x.to(torch.bfloat16).to(x.dtype) - x).detach()


@pytest.mark.parametrize("beta", [0.5, 1.0])
def test_aluglu_matches_oracle(beta):
    from algx.layers import aluglu
    g = torch.Generator().manual_seed(13)
    rows, ff = 257, 2048
    gu = (torch.randn((rows, 2 * ff), generator=g) * 3).to(torch.bfloat16)
    gu[0, ff:ff + 6] = torch.tensor([-3000.0, -300.0, -30.0, 0.0, 30.0, 300.0]).to(torch.bfloat16)
    dy = torch.randn((rows, ff), generator=g).to(torch.bfloat16)
    x = gu.cuda().requires_grad_(True)
    y = aluglu(x, beta)
    y.backward(dy.cuda())
    # reference rounding points: act = bf16(alu(up)), y = bf16(gate * act),
    # d(act) = bf16(dy * gate), dgate = bf16(dy * act)
    gf = gu.double().requires_grad_(True)
    gate, up = gf[:, :ff], gf[:, ff:]
    act = R.alu(up, beta, io_dtype=torch.bfloat16)
    ref = _rb(gate * act)
    ref.backward(dy.double())
    yr = ref.detach()
    assert torch.all((y.detach().cpu().double() - yr).abs() <= 2.0 ** -7 * yr.abs() + 1e-30)
    assert _rel_l2(x.grad.cpu(), gf.grad) < 1e-2
    assert torch.isfinite(x.grad.float()).all()


class _AlgLikelihood(torch.autograd.Function):
    """The alg_ce objective with the reference's custom VJP (algebraic.py:231-262)."""

    @staticmethod
    def forward(ctx, z, targets, n, c):
        ctx.save_for_backward(z, targets)
        ctx.n, ctx.c = n, c
        obj, _ = R.algebraic_likelihood(z.detach(), targets, n, c)
        return obj

    @staticmethod
    def backward(ctx, g):
        z, targets = ctx.saved_tensors
        return R.algebraic_likelihood_grad(z, targets, ctx.n, ctx.c, float(g)), None, None, None


def _restated_algebraic_loss(cfg, params, tokens, targets):
    """model.py:184-226 for the algebraic preset in float64, bf16 rounding points as the model."""
    B, T = tokens.shape
    d, H, D = cfg.d_model, cfg.n_heads, cfg.head_dim
    P = lambda n: params[n]  # noqa: E731
    cos, sin = R.cayley_table_geometric(D, T, cfg.rope_base, dtype=F64)
    x = _rb(P("embed")[tokens])
    x = R.rms_norm(x, P("embed_gain"), cfg.eps, io_dtype=torch.bfloat16)
    for i in range(cfg.n_layers):
        p = lambda n: P(f"layers.{i}.{n}")  # noqa: E731
        h = R.rms_norm(x, p("ln1"), cfg.eps, io_dtype=torch.bfloat16)
        qkv = _rb(h @ _rb(p("w_qkv")))
        q, k, v = (qkv[..., j * d:(j + 1) * d].reshape(B, T, H, D).transpose(1, 2) for j in range(3))
        q = R.rms_norm(q, p("q_gain"), cfg.eps, io_dtype=torch.bfloat16)
        k = R.rms_norm(k, p("k_gain"), cfg.eps, io_dtype=torch.bfloat16)
        q = R.apply_rotary(q, cos, sin, io_dtype=torch.bfloat16)
        k = R.apply_rotary(k, cos, sin, io_dtype=torch.bfloat16)
        sink = p("sink")[None, :, None, None]
        a = R.asinh_attention(q, k, v, n=cfg.attn_n, c=cfg.attn_c, sink_logit=sink, io_dtype=torch.bfloat16)
        a = a.transpose(1, 2).reshape(B, T, d)
        x = _rb(x + _rb(a @ _rb(p("w_o"))))
        h2 = R.rms_norm(x, p("ln2"), cfg.eps, io_dtype=torch.bfloat16)
        gu = _rb(h2 @ _rb(p("w_gu")))
        gate, up = gu[..., :cfg.d_ff], gu[..., cfg.d_ff:]
        act = _rb(gate * R.alu(up, cfg.alu_beta, io_dtype=torch.bfloat16))
        x = _rb(x + _rb(act @ _rb(p("w_d"))))
    hid = R.rms_norm(x, P("final_gain"), cfg.eps, io_dtype=torch.bfloat16)
    z = hid.reshape(B * T, d) @ _rb(P("embed")).T
    return _AlgLikelihood.apply(z, targets.reshape(-1), cfg.head_n, cfg.head_c)


def test_algebraic_preset_model_matches_float64_restatement():
    from algx.model import AlgebraicLM, config_algebraic_125m
    cfg = config_algebraic_125m(vocab_size=1000, d_model=128, n_layers=2, n_heads=2, d_ff=256, seq_len=256)
    model = AlgebraicLM(cfg, device="cuda", seed=3)
    with torch.no_grad():  # a non-zero sink so its gradient path is exercised
        model.flat["layers.0.sink"].copy_(torch.tensor([0.3, -0.2]))
        model.flat["layers.1.sink"].copy_(torch.tensor([-0.1, 0.25]))
    g = torch.Generator().manual_seed(9)
    seq = torch.randint(0, cfg.vocab_size, (2, cfg.seq_len + 1), generator=g)
    tok, tgt = seq[:, :-1].contiguous(), seq[:, 1:].contiguous()
    model.flat.zero_grad()
    obj, _ = model.loss(tok.cuda(), tgt.cuda())
    obj.backward()
    torch.cuda.synchronize()
    params = {n: p.detach().cpu().double().requires_grad_(True) for n, p in model.flat.params.items()}
    ref = _restated_algebraic_loss(cfg, params, tok, tgt)
    ref.backward()
    assert abs(float(obj) - float(ref)) <= 2e-3 * abs(float(ref)), (float(obj), float(ref))
    bad = {}
    for n, p in model.flat.params.items():
        err = _rel_l2(p.grad.cpu(), params[n].grad)
        if err > 3e-2:
            bad[n] = err
    assert not bad, bad
    from algx import _lib as L
    assert L.device_error() == 0
