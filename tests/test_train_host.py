"""Host logic of the config-5 training step (no GPU): the parameter layout of
algx.model and the data-parallel step of algx.train on gloo CPU ranks.

The step is generic over a module exposing ``flat`` and ``loss``; here a toy
model made of torch CPU ops stands in for the CUDA model, so these tests
check only the accumulation, bucketed all-reduce, clipping and AdamW logic.
"""

import math
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from algx import model as M
from algx.train import DataParallelTrainer


def test_125m_parameter_count_and_flops():
    cfg = M.config_125m()
    # tied embedding 50304 x 768, 12 blocks of 4 d^2 + 3 d f, gains (model.py:84-117)
    assert M.count_params(cfg) == 123_589_632
    # 6 P + 6 L S d = 741.54 M + 113.25 M per token; 112.0 TFLOP per 131072-token step
    assert abs(M.train_flops_per_token(cfg) - 854.784e6) < 1e3
    assert abs(M.train_flops_per_token(cfg) * 131072 / 1e12 - 112.04) < 0.01


def test_decay_mask_matches_reference_rule():
    # model.py:120-125: weight matrices (w_*) and the embedding decay; gains and sinks do not
    for sp in M.param_specs(M.config_125m(sink="learned")):
        leaf = sp.name.split(".")[-1]
        assert sp.decay == (leaf.startswith("w_") or leaf == "embed"), sp.name


def test_flat_params_share_storage_with_views():
    specs = M.param_specs(M.LMConfig(vocab_size=256, d_model=128, n_layers=2, n_heads=2, d_ff=256, seq_len=128))
    fp = M.FlatParams(specs, "cpu", torch.Generator().manual_seed(0))
    covered = {True: 0, False: 0}
    for sp in specs:
        p = fp[sp.name]
        decay, a, b = fp.slices[sp.name]
        covered[decay] += b - a
        assert p.data_ptr() == fp.data[decay][a:b].data_ptr()
        assert p.grad.data_ptr() == fp.grad[decay][a:b].data_ptr()
        if sp.std == 0:
            assert torch.all(p == sp.fill)
    assert covered[True] == fp.data[True].numel() and covered[False] == fp.data[False].numel()
    fp.flat[True].data.add_(1.0)  # an optimizer update of the flat tensor reaches every view
    assert torch.all(fp["final_gain"] == 1.0) and fp["embed"].data_ptr() == fp.data[True][
        fp.slices["embed"][1]:].data_ptr()


class ToyLM(torch.nn.Module):
    """Embedding -> RMS-free projection -> cross-entropy, in torch CPU ops, with FlatParams."""

    def __init__(self, seed=0):
        super().__init__()
        # three 12 x 12 matrices: a Muon stack that two ranks split unevenly
        specs = [M.ParamSpec("out_gain", (6,), False, 0.0, 1.0),
                 M.ParamSpec("w_b", (12, 6), True, 0.3),
                 M.ParamSpec("w_c", (12, 12), True, 0.3),
                 M.ParamSpec("w_e", (12, 12), True, 0.3),
                 M.ParamSpec("w_f", (12, 12), True, 0.3),
                 M.ParamSpec("w_a", (8, 12), True, 0.3),
                 M.ParamSpec("embed", (20, 8), True, 0.5)]
        self.flat = M.FlatParams(specs, "cpu", torch.Generator().manual_seed(seed))

    def loss(self, tokens, targets):
        x = torch.nn.functional.embedding(tokens, self.flat["embed"])
        h = torch.tanh(x @ self.flat["w_a"])
        h = h + 0.5 * (torch.tanh(h @ self.flat["w_c"]) + torch.tanh(h @ self.flat["w_e"]) -
                       torch.tanh(h @ self.flat["w_f"]))
        z = h @ self.flat["w_b"] * self.flat["out_gain"]
        nll = torch.nn.functional.cross_entropy(z.reshape(-1, 6), targets.reshape(-1), reduction="none")
        return nll.mean(), nll.detach()


def _batch():
    g = torch.Generator().manual_seed(3)
    seq = torch.randint(0, 20, (8, 17), generator=g)
    return seq[:, :-1], seq[:, 1:] % 6


def _run_single(steps=2, micro=2, clip=0.5, optimizer="adamw"):
    model = ToyLM()
    tr = DataParallelTrainer(model, lr=1e-2, micro_batch=micro, clip=clip, optimizer=optimizer, total_steps=10)
    tok, tgt = _batch()
    losses = [float(tr.step(tok, tgt)) for _ in range(steps)]
    return losses, {k: v.clone() for k, v in model.flat.data.items()}


def test_accumulation_equals_one_pass():
    """Micro-batches of 2 accumulate to the same step as one pass over all 8 sequences."""
    l1, p1 = _run_single(micro=2)
    l2, p2 = _run_single(micro=8)
    assert all(abs(a - b) < 1e-6 for a, b in zip(l1, l2))
    for k in p1:
        torch.testing.assert_close(p1[k], p2[k], rtol=1e-5, atol=1e-6)


def test_clip_scales_to_the_bound():
    model = ToyLM()
    tr = DataParallelTrainer(model, lr=0.0, micro_batch=8, clip=1e-3, weight_decay=0.0)
    tok, tgt = _batch()
    tr.step(tok, tgt)
    g = torch.cat([v.flatten() for v in model.flat.grad.values()])
    assert float(tr.last_gnorm) > 1e-3
    assert abs(float(torch.linalg.vector_norm(g)) - 1e-3) < 1e-8


def _worker(rank, world, init_file, q, shard=True, optimizer="adamw"):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "algebraic-extra_b200")]
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        from algx.train import DataParallelTrainer as T
        from tests.test_train_host import ToyLM, _batch
        model = ToyLM()
        # small buckets: several exchanges per step, launched from the backward hooks
        tr = T(model, lr=1e-2, micro_batch=2, clip=0.5, bucket_bytes=256, shard_optimizer=shard,
               optimizer=optimizer, total_steps=10)
        tok, tgt = _batch()
        per = tok.shape[0] // world
        sl = slice(rank * per, (rank + 1) * per)
        losses = [float(tr.step(tok[sl], tgt[sl])) for _ in range(2)]
        nshard = len(tr._shard)
        nsplit = tr._ref_opt.sharded_groups if tr._ref_opt is not None else 0
        tr.close()  # waits for the last step's gathers of the updated slices
        # numpy copies: torch tensors would be shared by file descriptor and vanish with the process
        q.put((rank, len(tr._buckets), nshard, nsplit, losses,
               {k: v.numpy().copy() for k, v in model.flat.data.items()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shard,optimizer", [(True, "adamw"), (False, "adamw"), (True, "hybrid_muon_cadamw"),
                                             (True, "muon_adamw"), (False, "muon_adamw")],
                         ids=["sharded_optimizer", "replicated_optimizer", "hybrid_muon_cadamw", "muon_adamw",
                              "muon_adamw_replicated"])
def test_two_ranks_match_one_process(shard, optimizer):
    """2 gloo ranks with half the batch each give the single-process step on the
    whole batch, with the decayed parameters' update sharded over the ranks
    (reduce-scatter, AdamW on each rank's slice, in-place all-gather fenced on
    first use by the next forward), with the replicated update, and with the
    reference trainer's Muon optimizers: the three 12 x 12 matrices split over
    the ranks (two and one, plus a zero row) and all-gathered, or replicated."""
    ref_losses, ref = _run_single(micro=2, optimizer=optimizer)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init = os.path.join(tmp, "init")
        procs = [ctx.Process(target=_worker, args=(r, 2, init, q, shard, optimizer)) for r in range(2)]
        for p in procs:
            p.start()
        out = [q.get(timeout=120) for _ in procs]
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    for rank, nb, nshard, nsplit, losses, params in out:
        assert nb >= 3
        assert (nshard >= 2) if (shard and optimizer == "adamw") else nshard == 0
        assert nsplit == (1 if (shard and optimizer != "adamw") else 0)
        assert all(abs(a - b) < 1e-6 for a, b in zip(losses, ref_losses)), (losses, ref_losses)
        for k in ref:
            torch.testing.assert_close(torch.from_numpy(params[k]), ref[k], rtol=1e-5, atol=1e-6)


def test_optimizer_step_bumps_the_version_of_every_view():
    """The model's bf16 weight copies are keyed on the master's version: an
    optimizer update of the flat buffer must change each view's version."""
    specs = M.param_specs(M.LMConfig(vocab_size=256, d_model=128, n_layers=1, n_heads=2, d_ff=256, seq_len=128))
    fp = M.FlatParams(specs, "cpu", torch.Generator().manual_seed(0))
    before = {n: p._version for n, p in fp.params.items()}
    opt = torch.optim.AdamW([fp.flat[True], fp.flat[False]], lr=1e-3)
    for k in (True, False):
        fp.flat[k].grad = torch.ones_like(fp.flat[k])
    opt.step()
    assert all(fp.params[n]._version != v for n, v in before.items())


def test_parse_overrides_types_values_like_the_reference_cli():
    over = M.parse_overrides(["n_layers=2", "attn_c=4", "head=alg_ce", "d_model=128"])
    assert over == {"n_layers": 2, "attn_c": 4.0, "head": "alg_ce", "d_model": 128}
    assert isinstance(over["attn_c"], float) and isinstance(over["n_layers"], int)
    cfg = M.config_125m(**over)
    assert cfg.n_layers == 2 and cfg.head == "alg_ce"
    with pytest.raises(ValueError, match="unknown config field"):
        M.parse_overrides(["heads=3"])


def test_check_finite_raises_before_the_update():
    """A non-finite loss raises FloatingPointError and leaves the masters untouched."""
    model = ToyLM()
    tr = DataParallelTrainer(model, lr=1e-2, micro_batch=8, check_finite=True)
    tok, tgt = _batch()
    tr.step(tok, tgt)  # finite: applied
    with torch.no_grad():
        model.flat["out_gain"][0] = float("nan")
    before = {k: v.clone() for k, v in model.flat.data.items()}
    with pytest.raises(FloatingPointError, match="not applied"):
        tr.step(tok, tgt)
    for k, v in model.flat.data.items():
        assert torch.allclose(v, before[k], equal_nan=True)


def _leaving_worker(rank, init_file, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "algebraic-extra_b200")]
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=10))
    if rank == 1:  # leaves between steps, before joining any collective
        dist.destroy_process_group()
        q.put((rank, "left"))
        return
    try:
        from algx.train import DataParallelTrainer as T
        from tests.test_train_host import ToyLM, _batch
        tr = T(ToyLM(), lr=1e-2, micro_batch=2, bucket_bytes=256)
        tok, tgt = _batch()
        tr.step(tok[:4], tgt[:4])
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - the failure is the expected outcome
        q.put((rank, type(e).__name__))


def test_step_fails_instead_of_hanging_when_a_rank_leaves():
    """A rank that leaves before the step: the other rank's gradient all-reduce
    errors out (peer gone or process-group timeout) rather than waiting forever."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        init = os.path.join(tmp, "init")
        procs = [ctx.Process(target=_leaving_worker, args=(r, init, q)) for r in range(2)]
        for p in procs:
            p.start()
        out = dict(q.get(timeout=120) for _ in procs)
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert out[1] == "left"
    assert out[0] == "RuntimeError", out
