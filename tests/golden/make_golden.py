"""Generate golden fixtures by running the reference's own dense maths.

Runs in the build container only (it needs the reference checkout; pass its
root with ``--reference``). JAX is not installed here, so the reference's
``src/algebraic/algebraic.py``, ``standard.py`` and ``evaluation.py`` are
imported unchanged on top of ``tests/golden/jax_on_torch`` (a torch-CPU
stand-in for the JAX calls they make). Forward values come from the
reference's code; gradients come from torch autograd through that code, or
from the reference's own ``custom_vjp`` rules where it defines them.

Two precisions per case:
  * ``f64``: float64 end to end (the reference's x64 CPU test setting);
  * ``bf16``: bfloat16 I/O with float32 internals, reproducing the
    reference's rounding points (``p.astype(v.dtype)``, ``out.astype(q.dtype)``).

Usage: python tests/golden/make_golden.py --reference <path-to-reference-checkout>
Outputs: tests/golden/reference_dense.npz, reference_alu.npz and
reference_optim.npz (small; inputs are regenerated from seeds; ``--which``
writes one of them).
"""

import argparse
import hashlib
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "jax_on_torch"))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases  # noqa: E402


def _sha(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()[:16]


def _np(t):
    return t.detach().to(torch.float64).numpy().astype(np.float32)


def attention_goldens(RA, out):
    for idx, (name, n, c, with_sink, scale) in enumerate(cases.ATTN_CASES):
        seed = 100 + 10 * idx
        q, k, v, g, sink = cases.attn_inputs(seed, scale=scale, with_sink=with_sink)
        for prec in ("f64", "bf16"):
            io = torch.bfloat16 if prec == "bf16" else torch.float64
            leaves = [torch.from_numpy(a).to(io).requires_grad_(True) for a in (q, k, v)]
            s = None
            if with_sink:
                s = torch.from_numpy(sink).to(torch.float64 if prec == "f64" else torch.float32)
                s.requires_grad_(True)
            o = RA.asinh_attention(*leaves, n=n, c=c, sink_logit=s)
            gg = torch.from_numpy(g).to(torch.float64 if prec == "f64" else torch.float32)
            torch.sum(o.to(gg.dtype) * gg).backward()
            key = f"attn_{name}_{prec}"
            out[key + "_o"] = _np(o)
            for nm, t in zip(("dq", "dk", "dv"), leaves):
                out[key + "_" + nm] = _np(t.grad)
            if with_sink:
                out[key + "_dsink"] = _np(s.grad)
        out[f"attn_{name}_checksum"] = np.float64(sum(float(np.sum(a, dtype=np.float64))
                                                      for a in (q, k, v, g)))


def norm_goldens(RA, out):
    x, gain, dy = cases.norm_inputs(7)
    for eps in (1e-5, 1e-3):
        for prec in ("f64", "bf16"):
            io = torch.bfloat16 if prec == "bf16" else torch.float64
            xt = torch.from_numpy(x).to(io).requires_grad_(True)
            gt = torch.from_numpy(gain).to(torch.float64 if prec == "f64" else torch.float32)
            gt.requires_grad_(True)
            y = RA.rms_norm(xt, gt, eps)
            d = torch.from_numpy(dy).to(torch.float64 if prec == "f64" else torch.float32)
            torch.sum(y.to(d.dtype) * d).backward()
            key = f"norm_eps{eps:g}_{prec}"
            out[key + "_y"] = _np(y)
            out[key + "_dx"] = _np(xt.grad)
            out[key + "_dgain"] = _np(gt.grad)
    out["norm_checksum"] = np.float64(sum(float(np.sum(a, dtype=np.float64)) for a in (x, gain, dy)))


def likelihood_goldens(RA, RS, RE, out):
    z = torch.from_numpy(cases.normal(21, (7, 300), 6.0)).double()
    t = torch.tensor([0, 5, 299, 17, 17, 100, -100])      # -100: JAX wraps to column 200
    for n, c in ((16, 16.0), (8, 2.0)):
        key = f"lik_n{n}c{c:g}"
        zz = z.clone().requires_grad_(True)
        obj, pt = RA.algebraic_likelihood(zz, t, n, c)
        obj.backward()
        out[key + "_obj"] = np.float64(obj.item())
        out[key + "_pt"] = pt.detach().numpy()
        out[key + "_grad"] = zz.grad.numpy()
        zz = z.clone().requires_grad_(True)
        obj, pt = RA.algebraic_likelihood_lean(zz, t, n, c)
        out[key + "_lean_obj"] = np.float64(obj.item())
        out[key + "_lean_pt"] = pt.detach().numpy()
        out[key + "_logprob"] = RE.logprob_from_logits(z, t, "alg_ce", n, c).numpy()
    zz = z.clone().requires_grad_(True)
    obj, nll = RS.cross_entropy(zz, t)
    obj.backward()
    out["ce_obj"] = np.float64(obj.item())
    out["ce_nll"] = nll.numpy()
    out["ce_grad"] = zz.grad.numpy()


def head_goldens(RA, RS, out):
    """Dense head as the reference's fused-head tests define it (test_fused_head_tpu.py:23-25)."""
    h, e, t = cases.head_inputs(31)
    tt = torch.from_numpy(t)
    for prec in ("f64", "bf16"):
        io = torch.bfloat16 if prec == "bf16" else torch.float64
        for kind, n, c in (("alg_ce", 8, 2.0), ("alg_ce", 16, 16.0), ("ce", 0, 0.0)):
            ht = torch.from_numpy(h).to(io).requires_grad_(True)
            et = torch.from_numpy(e).to(torch.float64 if prec == "f64" else torch.float32)
            et.requires_grad_(True)
            jnp = importlib.import_module("jax.numpy")
            z = jnp.matmul(ht, et.astype(ht.dtype).T, preferred_element_type=jnp.float32)
            if kind == "ce":
                obj, tel = RS.cross_entropy(z, tt)
                key = f"head_ce_{prec}"
            else:
                obj, tel = RA.algebraic_likelihood(z, tt, n, c)
                key = f"head_alg_n{n}c{c:g}_{prec}"
            obj.backward()
            out[key + "_obj"] = np.float64(obj.item())
            out[key + "_tel"] = _np(tel)
            out[key + "_dh"] = _np(ht.grad)
            out[key + "_de"] = _np(et.grad)
    out["head_checksum"] = np.float64(float(np.sum(h, dtype=np.float64)) +
                                      float(np.sum(e, dtype=np.float64)) + float(t.sum()))


def alu_goldens(RA, out):
    """alu(x, beta) (algebraic.py:86-101) and its custom VJP (algebraic.py:104-113)
    through the reference's own code, float64 and bf16 I/O, both signs and the
    far negative tail that the r^2 / (1 - u) branch protects."""
    x = cases.normal(41, (6, 256), 4.0)
    x[0, :8] = np.array([0.0, -1e-3, 1e-3, -30.0, 30.0, -300.0, 300.0, -3000.0], dtype=np.float32)
    g = cases.normal(42, (6, 256))
    for beta in (0.5, 1.0):
        for prec in ("f64", "bf16"):
            io = torch.bfloat16 if prec == "bf16" else torch.float64
            xt = torch.from_numpy(x).to(io).requires_grad_(True)
            y = RA.alu(xt, beta)
            y.backward(torch.from_numpy(g).to(io))
            key = f"alu_b{beta:g}_{prec}"
            out[key + "_y"] = _np(y)
            out[key + "_dx"] = _np(xt.grad)
    out["alu_checksum"] = np.float64(float(np.sum(x, dtype=np.float64)) + float(np.sum(g, dtype=np.float64)))


def optim_goldens(RO, out):
    """newton_schulz_5, the cosine schedule and three steps of each optimizer
    (optimizers.py:27-62, 96-116, 118-240) through the reference's own code,
    float64 end to end."""
    for i, shape in enumerate(cases.OPTIM_NS_SHAPES):
        g = torch.from_numpy(cases.normal(61 + i, shape)).double()
        out["ns5_" + "x".join(map(str, shape)) + "_in"] = g.numpy()
        out["ns5_" + "x".join(map(str, shape))] = RO.newton_schulz_5(g).numpy()
    sched = RO.make_cosine_schedule(2e-2, 10, 0.2, 0.1)
    out["schedule"] = np.array([float(sched(torch.tensor(t))) for t in range(13)])
    params0, grads = cases.optim_inputs(71)
    mask = {k: torch.tensor(v) for k, v in cases.OPTIM_DECAY.items()}
    for name in ("muon_adamw", "cadamw", "hybrid_muon_cadamw"):
        init_fn, step_fn = RO.get_optimizer(name, **cases.OPTIM_ARGS)
        params = {k: torch.from_numpy(v).double() for k, v in params0.items()}
        state = init_fn(params)
        for step, gr in enumerate(grads):
            params, state = step_fn(step, params, {k: torch.from_numpy(v).double() for k, v in gr.items()}, state,
                                    mask)
            for k, v in params.items():
                out[f"opt_{name}_step{step}_{k}"] = v.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout")
    ap.add_argument("--which", choices=("all", "dense", "alu", "optim"), default="all",
                    help="dense: reference_dense.npz; alu: reference_alu.npz; optim: reference_optim.npz")
    args = ap.parse_args()
    src = os.path.join(args.reference, "src")
    sys.path.insert(0, src)
    RA = importlib.import_module("algebraic.algebraic")
    RS = importlib.import_module("algebraic.standard")
    RE = importlib.import_module("algebraic.evaluation")
    prov = {name: _sha(os.path.join(src, "algebraic", name))
            for name in ("algebraic.py", "standard.py", "evaluation.py")}
    torch.set_num_threads(8)
    if args.which in ("all", "dense"):
        out = {"provenance": np.array(repr(prov))}
        attention_goldens(RA, out)
        norm_goldens(RA, out)
        likelihood_goldens(RA, RS, RE, out)
        head_goldens(RA, RS, out)
        path = os.path.join(HERE, "reference_dense.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1e6:.2f} MB; {prov}")
    if args.which in ("all", "optim"):
        RO = importlib.import_module("algebraic.optimizers")
        oprov = {"optimizers.py": _sha(os.path.join(src, "algebraic", "optimizers.py"))}
        out = {"provenance": np.array(repr(oprov))}
        optim_goldens(RO, out)
        path = os.path.join(HERE, "reference_optim.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1e6:.2f} MB; {oprov}")
    if args.which in ("all", "alu"):
        out = {"provenance": np.array(repr(prov))}
        alu_goldens(RA, out)
        path = os.path.join(HERE, "reference_alu.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1e6:.2f} MB; {prov}")


if __name__ == "__main__":
    main()
