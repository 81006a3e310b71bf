"""Helpers shared by the GPU parity tests (kernel vs CPU oracle)."""

import os

import numpy as np
import torch

from oracle import reference_math as R


def rel_l2(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float(torch.linalg.norm(a - b) / max(float(torch.linalg.norm(b)), 1e-30))


def dump(name, **arrays):
    """Save arrays for offline diagnosis when ALGX_DUMP_DIR is set."""
    d = os.environ.get("ALGX_DUMP_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        np.savez(os.path.join(d, name + ".npz"),
                 **{k: torch.as_tensor(v).detach().float().cpu().numpy() for k, v in arrays.items()})


def algx_attention(fn, q, k, v, g, sink):
    """Run ``fn`` (the algx flash_attention with options bound) forward + backward."""
    leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]
    s = None if sink is None else sink.detach().clone().requires_grad_(True)
    o = fn(*leaves, s)
    torch.sum(o.float() * g.float()).backward()
    torch.cuda.synchronize()
    return o.detach(), leaves[0].grad, leaves[1].grad, leaves[2].grad, None if s is None else s.grad


def oracle_attention(q, k, v, g, sink, io_dtype=None, **opts):
    """Float64 CPU oracle of flash_attention on the same (rounded) inputs."""
    cpu = lambda t: None if t is None else t.detach().double().cpu()
    fn = lambda q_, k_, v_, s_: R.flash_attention(q_, k_, v_, s_, io_dtype=io_dtype, **opts)
    return R.attention_grads(fn, cpu(q), cpu(k), cpu(v), cpu(g), cpu(sink))
