"""GPU parity of the config-5 training step pieces: the row RMS norm and SwiGLU
kernels against the float64 oracle / fp32 formulas, the model's loss and
gradients against a float64 restatement of model.py with the same bf16
rounding points, and the data-parallel step itself.

Tolerances: RMS norm outputs within one bf16 ulp (fp32 I/O: 2e-6 relative),
gradients within 1e-2 relative L2 (bf16) / 1e-5 (fp32); SwiGLU within one
bf16 ulp forward and 1e-2 relative L2 backward; the 2-layer model's loss
within 2e-3 relative and each parameter gradient within 3e-2 relative L2 of
the restatement (bf16 activations through two blocks and the head).
"""

import math

import pytest
import torch

from oracle import reference_math as R

pytestmark = pytest.mark.gpu

F64 = torch.float64


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-300))


@pytest.mark.parametrize("dtype,dim,rows", [(torch.bfloat16, 768, 1000), (torch.bfloat16, 1024, 37),
                                            (torch.float32, 768, 515), (torch.bfloat16, 136, 64)])
def test_rmsnorm_matches_oracle(dtype, dim, rows):
    from algx.layers import rms_norm
    g = torch.Generator().manual_seed(dim + rows)
    x = (torch.randn((rows, dim), generator=g) * 3).to(dtype)
    gain = 1 + 0.1 * torch.randn(dim, generator=g)
    dy = torch.randn((rows, dim), generator=g).to(dtype)
    xc, gc = x.cuda().requires_grad_(True), gain.cuda().requires_grad_(True)
    y = rms_norm(xc, gc, 1e-5)
    y.backward(dy.cuda())
    ref = R.rms_norm(x.double(), gain.double(), 1e-5, io_dtype=dtype)
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2e-6
    assert torch.all((y.cpu().double() - ref).abs() <= ulp * ref.abs() + 1e-30)
    dx, dgain = R.qk_norm_backward(x.double(), gain.double(), dy.double(), 1e-5)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel_l2(xc.grad.cpu(), dx) < tol
    assert _rel_l2(gc.grad.cpu(), dgain) < 1e-5


def test_rmsnorm_without_gain_and_empty():
    from algx.layers import rms_norm
    x = torch.randn((64, 256), device="cuda").to(torch.bfloat16).requires_grad_(True)
    y = rms_norm(x, None)
    ref = R.rms_norm(x.detach().cpu().double(), None, 1e-5, io_dtype=torch.bfloat16)
    assert torch.all((y.detach().cpu().double() - ref).abs() <= 2.0 ** -7 * ref.abs())
    y.sum().backward()
    assert torch.isfinite(x.grad.float()).all()
    e = torch.empty((0, 768), device="cuda", dtype=torch.bfloat16)
    assert rms_norm(e, torch.ones(768, device="cuda")).shape == (0, 768)


def test_swiglu_matches_fp32_formula():
    from algx.layers import swiglu
    g = torch.Generator().manual_seed(11)
    rows, ff = 300, 2048
    gu = (torch.randn((rows, 2 * ff), generator=g) * 2).to(torch.bfloat16)
    dy = torch.randn((rows, ff), generator=g).to(torch.bfloat16)
    x = gu.cuda().requires_grad_(True)
    y = swiglu(x)
    y.backward(dy.cuda())
    gf = gu.double().requires_grad_(True)
    gate, up = gf[:, :ff], gf[:, ff:]
    ref = gate * (up * torch.sigmoid(up))
    ref.backward(dy.double())
    yr = ref.detach().to(torch.bfloat16).double()
    assert torch.all((y.detach().cpu().double() - yr).abs() <= 2.0 ** -7 * yr.abs() + 1e-6)
    assert _rel_l2(x.grad.cpu(), gf.grad) < 1e-2


def _tiny_cfg(**kw):
    from algx.model import LMConfig
    base = dict(vocab_size=1000, d_model=128, n_layers=2, n_heads=2, d_ff=256, seq_len=256)
    base.update(kw)
    return LMConfig(**base)


def _rb(x):
    """Straight-through bf16 rounding (the reference's .astype(bf16) points)."""
    return x + (x.to(torch.bfloat16).to(x.dtype) - x).detach()


def _restated_loss(cfg, params, tokens, targets):
    """model.py:184-226 in float64 with bf16 rounding of every stored activation."""
    B, T = tokens.shape
    d, H, D = cfg.d_model, cfg.n_heads, cfg.head_dim
    P = lambda n: params[n]  # noqa: E731
    cos, sin = R.rope_table(D, T, cfg.rope_base, dtype=F64)
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
        a = R.asinh_attention(q, k, v, n=cfg.attn_n, c=cfg.attn_c, io_dtype=torch.bfloat16)
        a = a.transpose(1, 2).reshape(B, T, d)
        x = _rb(x + _rb(a @ _rb(p("w_o"))))
        h2 = R.rms_norm(x, p("ln2"), cfg.eps, io_dtype=torch.bfloat16)
        gu = _rb(h2 @ _rb(p("w_gu")))
        gate, up = gu[..., :cfg.d_ff], gu[..., cfg.d_ff:]
        act = _rb(gate * (up * torch.sigmoid(up)))
        x = _rb(x + _rb(act @ _rb(p("w_d"))))
    hid = R.rms_norm(x, P("final_gain"), cfg.eps, io_dtype=torch.bfloat16)
    z = hid.reshape(B * T, d) @ _rb(P("embed")).T
    obj, _ = R.cross_entropy(z, targets.reshape(-1))
    return obj


def test_model_matches_float64_restatement():
    from algx.model import AlgebraicLM
    cfg = _tiny_cfg()
    model = AlgebraicLM(cfg, device="cuda", seed=0)
    g = torch.Generator().manual_seed(5)
    seq = torch.randint(0, cfg.vocab_size, (2, cfg.seq_len + 1), generator=g)
    tok, tgt = seq[:, :-1].contiguous(), seq[:, 1:].contiguous()
    model.flat.zero_grad()
    obj, _ = model.loss(tok.cuda(), tgt.cuda())
    obj.backward()
    torch.cuda.synchronize()
    params = {n: p.detach().cpu().double().requires_grad_(True) for n, p in model.flat.params.items()}
    ref = _restated_loss(cfg, params, tok, tgt)
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


def test_train_step_reduces_loss_on_a_fixed_batch():
    from algx.model import AlgebraicLM
    from algx.train import DataParallelTrainer
    cfg = _tiny_cfg(sink="learned")
    model = AlgebraicLM(cfg, device="cuda", seed=1)
    tr = DataParallelTrainer(model, lr=3e-3, micro_batch=2)
    g = torch.Generator(device="cuda").manual_seed(2)
    seq = torch.randint(0, cfg.vocab_size, (4, cfg.seq_len + 1), device="cuda", generator=g)
    tok, tgt = seq[:, :-1].contiguous(), seq[:, 1:].contiguous()
    before = model.flat.data[True].clone()
    losses = [float(tr.step(tok, tgt)) for _ in range(6)]
    assert all(math.isfinite(l) for l in losses)
    assert losses[-1] < losses[0] - 0.05, losses
    assert not torch.equal(before, model.flat.data[True])
    assert math.isfinite(float(tr.last_gnorm))
    from algx import _lib as L
    assert L.device_error() == 0


def test_heads_tokens_permute_is_exact():
    from algx import _lib as L
    for dt in (torch.bfloat16, torch.float32):
        B, H, T, D = 3, 5, 384, 64
        x = torch.randn((B, H, T, D), device="cuda").to(dt)
        tok = torch.empty((B, T, H, D), device="cuda", dtype=dt)
        back = torch.empty_like(x)
        lib = L.lib()
        st = L.stream_of(x)
        L.check(lib.algx_heads_to_tokens(x.data_ptr(), tok.data_ptr(), B, H, T, D, L.dtype_code(dt), st), "h2t")
        L.check(lib.algx_tokens_to_heads(tok.data_ptr(), back.data_ptr(), B, H, T, D, L.dtype_code(dt), st), "t2h")
        assert torch.equal(tok, x.permute(0, 2, 1, 3))
        assert torch.equal(back, x)


@pytest.mark.parametrize("with_sink,T", [(False, 512), (True, 512), (False, 200)])
def test_packed_attention_matches_head_major(with_sink, T):
    """qknorm_flash_attention_packed on (B, T, 3, H, D) = transposes around
    qknorm_flash_attention: forward bit-identical, gradients within the
    run-to-run spread of the dQ reduce-adds (1e-3 relative L2). T = 200 (not
    a multiple of 128) runs on the CUDA-core kernels."""
    from algx.kernels.flash import qknorm_flash_attention, qknorm_flash_attention_packed
    from algx.rotary import rope_table
    B, H, D = 2, 3, 64
    g = torch.Generator(device="cuda").manual_seed(21)
    qkv = torch.randn((B, T, 3, H, D), device="cuda", generator=g).to(torch.bfloat16)
    gq = 1 + 0.05 * torch.randn(D, device="cuda", generator=g)
    gk = 1 + 0.05 * torch.randn(D, device="cuda", generator=g)
    sink = (0.3 * torch.randn(H, device="cuda", generator=g)) if with_sink else None
    do = torch.randn((B, T, H, D), device="cuda", generator=g).to(torch.bfloat16)
    rot = rope_table(D, T, device="cuda")
    kw = dict(eps=1e-5, kind="asinh", n=16, c=8.0, range_guard=True, rotary=rot)

    a = qkv.clone().requires_grad_(True)
    ga, gb = gq.clone().requires_grad_(True), gk.clone().requires_grad_(True)
    sa = sink.clone().requires_grad_(True) if with_sink else None
    o1 = qknorm_flash_attention_packed(a, ga, gb, sa, **kw)
    o1.backward(do)

    b_ = qkv.clone().requires_grad_(True)
    gc, gd = gq.clone().requires_grad_(True), gk.clone().requires_grad_(True)
    sb = sink.clone().requires_grad_(True) if with_sink else None
    q, k, v = (b_[:, :, j].permute(0, 2, 1, 3) for j in range(3))
    o2 = qknorm_flash_attention(q, k, v, gc, gd, sb, **kw).permute(0, 2, 1, 3)
    o2.backward(do)

    assert torch.equal(o1, o2)
    assert _rel_l2(a.grad, b_.grad) < 1e-3
    assert _rel_l2(ga.grad, gc.grad) < 1e-3 and _rel_l2(gb.grad, gd.grad) < 1e-3
    if with_sink:
        assert _rel_l2(sa.grad, sb.grad) < 1e-3
    from algx import _lib as L
    assert L.device_error() == 0


@pytest.mark.parametrize("dtype,dim", [(torch.bfloat16, 768), (torch.bfloat16, 1024), (torch.float32, 768)])
def test_add_rms_norm_matches_composed(dtype, dim):
    """The fused residual add + norm equals x + r followed by rms_norm: s and y
    bit-identical, gradients within one rounding (1e-2 / 1e-5 relative L2)."""
    from algx.layers import add_rms_norm, rms_norm
    g = torch.Generator(device="cuda").manual_seed(dim)
    x = torch.randn((777, dim), device="cuda", generator=g).to(dtype)
    r = torch.randn((777, dim), device="cuda", generator=g).to(dtype)
    gain = 1 + 0.1 * torch.randn(dim, device="cuda", generator=g)
    ds = torch.randn((777, dim), device="cuda", generator=g).to(dtype)
    dy = torch.randn((777, dim), device="cuda", generator=g).to(dtype)
    a = [t.clone().requires_grad_(True) for t in (x, r, gain)]
    s1, y1 = add_rms_norm(a[0], a[1], a[2], 1e-5)
    torch.autograd.backward([s1, y1], [ds, dy])
    b = [t.clone().requires_grad_(True) for t in (x, r, gain)]
    s2 = b[0] + b[1]
    y2 = rms_norm(s2, b[2], 1e-5)
    torch.autograd.backward([s2, y2], [ds, dy])
    assert torch.equal(s1, s2) and torch.equal(y1, y2)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel_l2(a[0].grad, b[0].grad) < tol and _rel_l2(a[1].grad, b[1].grad) < tol
    assert _rel_l2(a[2].grad, b[2].grad) < 1e-5


@pytest.mark.parametrize("name,precision,tol", [("muon_adamw", "highest", 1e-3),
                                                  ("hybrid_muon_cadamw", "highest", 1e-3),
                                                  ("hybrid_muon_cadamw", "default", 2e-2)])
def test_reference_optimizer_step_on_the_model_matches_float64(name, precision, tol):
    """One trainer step with the reference trainer's optimizer on the GPU
    (float32 masters; Newton-Schulz batched over same-shape matrices, with
    float32 or bf16 operands) against the same update of the same masters and
    clipped gradients replayed in float64 on the CPU with the same operand
    rounding. ``tol`` bounds the update's relative error: bf16 operands can
    round differently from float32 and float64 intermediates."""
    from algx import model as M
    from algx.optim import ReferenceOptimizer
    from algx.train import DataParallelTrainer
    cfg = M.config_125m(vocab_size=1000, d_model=128, n_layers=2, n_heads=2, d_ff=256, seq_len=256)
    model = M.AlgebraicLM(cfg, device="cuda", seed=1)
    tr = DataParallelTrainer(model, lr=2e-2, micro_batch=2, optimizer=name, total_steps=10,
                             opt_kwargs={"precision": precision})
    g = torch.Generator().manual_seed(12)
    seq = torch.randint(0, 1000, (2, 257), generator=g)
    before = {k: v.detach().double().cpu() for k, v in model.flat.params.items()}
    tr.step(seq[:, :-1].cuda(), seq[:, 1:].cuda())
    torch.cuda.synchronize()
    after = {k: v.detach().double().cpu() for k, v in model.flat.params.items()}
    ref = {k: v.clone() for k, v in before.items()}
    for k, v in ref.items():
        v.grad = model.flat.params[k].grad.detach().double().cpu()  # the clipped gradient the step used
    opt = ReferenceOptimizer(name, [(k, ref[k], model.flat.slices[k][0]) for k in ref], lr=2e-2, total_steps=10,
                             precision=precision)
    opt.step(0)
    num = sum(float(torch.sum((after[k] - ref[k]) ** 2)) for k in ref)
    den = sum(float(torch.sum((ref[k] - before[k]) ** 2)) for k in ref)
    assert den > 0 and (num / den) ** 0.5 < tol, (num, den)


def test_newton_schulz_bf16_operands_on_tensor_cores():
    """precision="default" on a CUDA float32 batch runs bf16 x bf16 -> float32
    products; against the float64 emulation (operands rounded to bf16) and
    the exact float64 orthogonalisation."""
    from algx.optim import newton_schulz_5
    g = torch.Generator().manual_seed(4)
    x = torch.randn(6, 256, 768, generator=g, dtype=torch.float64)
    got = newton_schulz_5(x.float().cuda(), precision="default").double().cpu()
    emul = newton_schulz_5(x, precision="default")
    exact = newton_schulz_5(x, precision="highest")
    rel = lambda a, b: float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
    assert rel(got, emul) < 1e-2 and rel(got, exact) < 3e-2, (rel(got, emul), rel(got, exact))
    assert rel(newton_schulz_5(x.float().cuda(), precision="highest").double().cpu(), exact) < 1e-4
