"""Data-parallel training step on two GPUs (NCCL): the sharded optimizer
(reduce-scatter, AdamW on each rank's slice, in-place all-gather fenced on
first use) gives the same losses and master weights as the replicated update
(all-reduce, AdamW on every rank), step after step; and the reference
trainer's hybrid Muon + cautious AdamW with its Muon matrices split over the
ranks (all-gathered after the update) as with every rank updating them all."""

import os
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu


def _train(rank, world, init_file, shard, q, optimizer):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "algebraic-extra_b200")]
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    try:
        from algx import model as M
        from algx.train import DataParallelTrainer
        cfg = M.config_125m(vocab_size=1000, d_model=128, n_layers=2, n_heads=2, d_ff=256, seq_len=256)
        model = M.AlgebraicLM(cfg, device="cuda", seed=5)
        tr = DataParallelTrainer(model, lr=1e-3, micro_batch=2, bucket_bytes=64 << 10, shard_optimizer=shard,
                                 optimizer=optimizer, total_steps=10)
        g = torch.Generator().manual_seed(11)
        seq = torch.randint(0, 1000, (8, 257), generator=g)
        per = seq.shape[0] // world
        tok, tgt = seq[rank * per:(rank + 1) * per, :-1].cuda(), seq[rank * per:(rank + 1) * per, 1:].cuda()
        losses = [float(tr.step(tok, tgt)) for _ in range(3)]
        nshard = len(tr._shard) if optimizer == "adamw" else tr._ref_opt.sharded_groups
        tr.close()
        torch.cuda.synchronize()
        q.put((rank, shard, nshard, losses, {k: v.cpu().numpy().copy() for k, v in model.flat.data.items()}))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("optimizer", ["adamw", "hybrid_muon_cadamw"])
def test_sharded_optimizer_matches_replicated_two_gpus(optimizer):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = {}
    for shard in (True, False):
        q = ctx.Queue()
        with tempfile.TemporaryDirectory() as tmp:
            procs = [ctx.Process(target=_train, args=(r, 2, os.path.join(tmp, "pg"), shard, q, optimizer))
                     for r in range(2)]
            for p in procs:
                p.start()
            res = [q.get(timeout=300) for _ in procs]
            for p in procs:
                p.join(timeout=120)
                assert p.exitcode == 0
        out[shard] = {r[0]: r for r in res}
    for rank in (0, 1):
        _, _, nshard, l_s, p_s = out[True][rank]
        _, _, n0, l_r, p_r = out[False][rank]
        assert nshard >= (2 if optimizer == "adamw" else 3) and n0 == 0
        assert all(abs(a - b) <= 1e-5 * abs(b) for a, b in zip(l_s, l_r)), (l_s, l_r)
        for k in p_r:
            torch.testing.assert_close(torch.from_numpy(p_s[k]), torch.from_numpy(p_r[k]), rtol=1e-5, atol=1e-6)
    # both ranks hold the same masters after the gathers
    for k in out[True][0][4]:
        torch.testing.assert_close(torch.from_numpy(out[True][0][4][k]), torch.from_numpy(out[True][1][4][k]),
                                   rtol=0, atol=0)
