"""The torch.library front-end: registration and shape inference without a GPU,
parity with the eager wrappers and tracing on the GPU."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import algx.torch_ops as T
from algx import _lib as L

OPS = ["qk_rms_norm", "qk_rms_norm_backward", "flash_attention_fwd", "flash_attention_bwd", "fused_head_fwd",
       "fused_head_bwd"]


@pytest.mark.parametrize("name", OPS)
def test_operator_registered(name):
    assert hasattr(torch.ops.algx, name)


def _fake(*shapes_dtypes):
    mode = FakeTensorMode()
    return mode, [mode.from_tensor(torch.empty(s, dtype=d)) for s, d in shapes_dtypes]


def test_fake_shapes_attention_and_norm():
    mode, (q, k, v, g) = _fake(((2, 3, 256, 64), torch.bfloat16), ((2, 3, 256, 64), torch.bfloat16),
                               ((2, 3, 256, 64), torch.bfloat16), ((64,), torch.float32))
    with mode:
        y = torch.ops.algx.qk_rms_norm(q, g, 1e-5)
        assert y.shape == q.shape and y.dtype == q.dtype
        guarded = [L.ALGX_ATTN_ASINH, L.ALGX_MODE_GUARDED, 16, 1, 1, 0]
        o, q_s, stat, guard, o_prec = torch.ops.algx.flash_attention_fwd(q, k, v, None, guarded,
                                                                       [63.75, 0.0625, 200.0, 15.8, 1e8])
        assert o.shape == q.shape and q_s.shape == q.shape
        assert stat.shape == (2, 3, 256) and stat.dtype == torch.float32
        assert guard.shape == (4,) and o_prec.shape == q.shape
        clipped = [L.ALGX_ATTN_ASINH, L.ALGX_MODE_CLIPPED, 16, 1, 1, 0]
        *_, o_prec = torch.ops.algx.flash_attention_fwd(q, k, v, None, clipped, [63.75, 0.0625, 0.0, 0.0, 0.0])
        assert o_prec.numel() == 0
        dq, dk, dv, dsink = torch.ops.algx.flash_attention_bwd(q_s, k, v, None, o, o_prec, stat, guard, o,
                                                               clipped, [63.75, 0.0625, 0.0, 0.0, 0.0])
        assert dq.shape == dk.shape == dv.shape == q.shape and dsink.numel() == 0


def test_fake_shapes_head():
    mode, (h, e, t) = _fake(((512, 128), torch.bfloat16), ((1000, 128), torch.float32), ((512,), torch.int32))
    with mode:
        obj, tel, stat, count = torch.ops.algx.fused_head_fwd(h, e, t, [L.ALGX_HEAD_CE, 16, 0, 0], [1.0, 0.0, 1.0])
        assert obj.shape == () and tel.shape == (512,) and stat.shape == (512,) and count.shape == (1,)
        dh, de = torch.ops.algx.fused_head_bwd(h, e, t, stat, count, [L.ALGX_HEAD_CE, 16, 0, 0], [1.0, 0.0, 1.0])
        assert dh.shape == h.shape and dh.dtype == h.dtype
        assert de.shape == e.shape and de.dtype == torch.float32


def test_export_keeps_opaque_nodes():
    """torch.export (dynamo) traces the wrappers on fake CUDA tensors, no GPU needed:
    each call stays one algx node and the configuration becomes constants."""

    class Block(torch.nn.Module):
        def forward(self, q, k, v, g, h, e, t):
            o = T.flash_attention(T.qk_rms_norm(q, g), k, v, kind="asinh", n=16, c=8., range_guard=True)
            obj, _ = T.fused_head(h, e, t, kind="alg_ce", n=8, c=2.)
            return o, obj

    with FakeTensorMode():
        qkv = [torch.empty((2, 3, 512, 64), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
        args = (*qkv, torch.empty(64, device="cuda"), torch.empty((512, 128), device="cuda"),
                torch.empty((1000, 128), device="cuda"), torch.empty(512, dtype=torch.int64, device="cuda"))
    ep = torch.export.export(Block(), args)
    algx_nodes = [n for n in ep.graph.nodes if n.op == "call_function" and "algx" in str(n.target)]
    assert [str(n.target) for n in algx_nodes] == ["algx.qk_rms_norm.default", "algx.flash_attention_fwd.default",
                                                   "algx.fused_head_fwd.default"]
    ints, floats = algx_nodes[1].args[4], algx_nodes[1].args[5]
    assert ints == [L.ALGX_ATTN_ASINH, L.ALGX_MODE_GUARDED, 16, 1, 1, 0]
    assert floats[1] == 1.0 / (8.0 * 8.0)
    assert algx_nodes[2].args[4][2] == 8 / 2.


def test_errors_match_eager_wrappers():
    q = torch.zeros((1, 1, 128, 32))
    with pytest.raises(ValueError, match="head_dim 64"):
        T.flash_attention(q, q, q, kind="asinh")
    with pytest.raises(ValueError, match="D=64"):
        T.qk_rms_norm(torch.zeros((8, 32)), torch.ones(64))
    with pytest.raises(ValueError, match="power of two"):
        T.fused_head(torch.zeros((8, 64)), torch.zeros((16, 64)), torch.zeros(8, dtype=torch.int64),
                     kind="alg_ce", n=6)


@pytest.mark.gpu
def test_ops_match_eager_and_trace():
    """Same values and gradients as algx.kernels; the whole block traces as opaque nodes."""
    from algx.kernels.flash import flash_attention as eager_flash
    from algx.kernels.fused_head import fused_head as eager_head
    from algx.kernels.qk_norm import qk_rms_norm as eager_norm
    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v, do = (torch.randn((2, 3, 512, 64), device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    gq = 1 + 0.02 * torch.randn(64, device="cuda", generator=g)

    def block(ops, q_, k_, v_, g_):
        return ops["flash"](ops["norm"](q_, g_), k_, v_, kind="asinh", n=16, c=8., range_guard=True)

    results = []
    for ops in ({"flash": eager_flash, "norm": eager_norm}, {"flash": T.flash_attention, "norm": T.qk_rms_norm}):
        leaves = [t.clone().requires_grad_(True) for t in (q, k, v, gq)]
        o = block(ops, *leaves)
        torch.sum(o.float() * do.float()).backward()
        results.append((o.detach(), [t.grad for t in leaves]))
    assert torch.equal(results[0][0], results[1][0])
    for a, b in zip(results[0][1], results[1][1]):
        assert float((a.float() - b.float()).norm() / b.float().norm()) < 1e-2
    compiled = torch.compile(lambda *a: block({"flash": T.flash_attention, "norm": T.qk_rms_norm}, *a),
                             backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled(q, k, v, gq), results[1][0])

    h = torch.randn((1024, 128), device="cuda", generator=g)
    e = 0.02 * torch.randn((4096, 128), device="cuda", generator=g)
    t = torch.randint(0, 4096, (1024,), device="cuda", generator=g)
    grads = []
    for fn in (eager_head, T.fused_head):
        hh, ee = h.clone().requires_grad_(True), e.clone().requires_grad_(True)
        obj, _ = fn(hh, ee, t, kind="ce")
        obj.backward()
        grads.append((obj.detach(), hh.grad, ee.grad))
    assert torch.allclose(grads[0][0], grads[1][0])
    for a, b in zip(grads[0][1:], grads[1][1:]):
        assert a.dtype == b.dtype and float((a - b).norm() / b.norm()) < 1e-6
