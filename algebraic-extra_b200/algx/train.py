"""Data-parallel training step: micro-batch accumulation, gradient all-reduce,
global-norm clipping and AdamW (train.py:265-290 of the reference).

One process per GPU. Each rank runs its share of the global batch as
micro-batches, accumulating float32 gradients in the model's flat gradient
buffers. During the last micro-batch's backward, each contiguous bucket of a
flat buffer is all-reduced (NCCL, asynchronously) as soon as autograd has
finished every parameter in it, so the exchange overlaps the rest of the
backward; the buffers are laid out in the order the backward finishes them.
Then, on the device and without a host synchronisation:

    g      = sum_ranks(g) / world                       (lax.pmean, train.py:281)
    gnorm  = ||g||_2
    g     *= min(1, clip / max(gnorm, 1e-12))           (train.py:283-285)
    AdamW on the two flat master buffers, weight decay on the decayed one only
    (model.py:120-125 mask)

With ``shard_optimizer`` (the default on more than one rank) the decayed
buckets are reduce-scattered instead of all-reduced: each rank receives the
summed gradient of its 1/world slice of every bucket, the global norm comes
from the slices' squared sums (one small all-reduce), AdamW updates only this
rank's slice of the float32 masters, and the updated slices are all-gathered
back in place, asynchronously and in the order the forward pass uses them;
the model's parameter lookup waits for a bucket's gather on first use, so the
gather overlaps the next forward. Gradient exchange volume is that of the
all-reduce; the update runs on 1/world of the decayed parameters. The
element-wise maths is unchanged, so the masters match the replicated update up
to the summation order of the gradient norm. Gains and sinks (the small
non-decayed buffer) and any bucket whose length is not a multiple of the world
size stay all-reduced and replicated.

The step works for any module that exposes ``flat`` (``algx.model.FlatParams``)
and ``loss(tokens, targets) -> (objective, telemetry)``; ``algx.model.AlgebraicLM``
is the one this package ships.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist


class DataParallelTrainer:
    """Train step over the ranks of ``group`` (all ranks when None).

    ``shard_optimizer``: shard the decayed parameters' update over the ranks
    (see the module docstring); ignored on one rank.
    ``optimizer``: "adamw" (fused AdamW with the constant ``lr``, the BASELINE
    configuration) or one of the reference trainer's optimizers,
    "muon_adamw", "cadamw", "hybrid_muon_cadamw" (``algx.optim``, with its
    cosine schedule over ``total_steps``; ``opt_kwargs`` go to it). With
    those the gradients are all-reduced whole; with ``shard_optimizer`` the
    ranks split the Muon matrices of each shape (Muon orthogonalises whole
    matrices) and all-gather the updated ones, and the rest of the update
    runs on every rank.

    ``micro_batch``: sequences per forward/backward pass; the rank's share of
    the batch must be a multiple of it. ``bucket_bytes``: target size of one
    all-reduce. ``check_finite``: before each optimizer update, read the loss
    and the gradient norm on the host and raise ``FloatingPointError`` if
    either is not finite (the reference trainer's check, train.py:423-427),
    leaving the master weights at their last finite values; it costs one host
    synchronisation per step, so it is off by default.
    """

    def __init__(self, model, *, lr: float = 2e-3, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1, clip: float = 1.0, micro_batch: int = 8,
                 bucket_bytes: int = 32 << 20, group=None, check_finite: bool = False,
                 shard_optimizer: bool = True, optimizer: str = "adamw", total_steps: int = 1000,
                 opt_kwargs: Optional[dict] = None):
        self.model = model
        self.check_finite = bool(check_finite)
        self.flat = model.flat
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        self.clip = float(clip)
        self.micro_batch = int(micro_batch)
        dev = self.flat.data[True].device
        self._works: List = []
        self._last = False
        self._buckets = self._make_buckets(bucket_bytes) if self.world > 1 else []
        self._ref_opt = None
        self._opt_step = 0
        if optimizer != "adamw":
            from .optim import ReferenceOptimizer
            named = [(n, p, self.flat.slices[n][0]) for n, p in self.flat.params.items()]
            # the gradients are all-reduced; with shard_optimizer the ranks
            # split the Newton-Schulz work and all-gather the updated matrices
            self._ref_opt = ReferenceOptimizer(optimizer, named, lr=lr, weight_decay=weight_decay,
                                               total_steps=total_steps, b1=betas[0], b2=betas[1], adam_eps=eps,
                                               shard=shard_optimizer and self.world > 1, group=group,
                                               **(opt_kwargs or {}))
            shard_optimizer = False
        # bucket index -> (this rank's slice of the masters, its gradient buffer)
        self._shard: Dict[int, Tuple[torch.Tensor, torch.Tensor]] = {}
        # bucket index -> the bucket's masters as a tensor on the same storage
        # with its own autograd version counter: the gather writes through it,
        # so finishing a gather (which gloo does at wait time) does not bump the
        # version of weights the forward has already saved for the backward.
        # Safe because every bucket is fenced before its first read, and the
        # model's bf16 weight copies are dropped when the gathers are issued.
        self._gather_out: Dict[int, torch.Tensor] = {}
        if shard_optimizer and self.world > 1:
            base = self.flat.data[True]
            for bi, (decay, a, b, _) in enumerate(self._buckets):
                if decay and (b - a) % self.world == 0:
                    n = (b - a) // self.world
                    lo = a + self.rank * n
                    self._shard[bi] = (base[lo:lo + n], torch.zeros(n, dtype=torch.float32, device=dev))
                    self._gather_out[bi] = torch.empty(0, dtype=base.dtype, device=dev).set_(
                        base.untyped_storage(), base.storage_offset() + a, (b - a,))
        if self._shard:
            decayed = []
            for bi, (decay, a, b, _) in enumerate(self._buckets):
                if not decay:
                    continue
                m, g = self._shard[bi] if bi in self._shard else (self.flat.data[True][a:b], self.flat.grad[True][a:b])
                p = torch.nn.Parameter(m)
                p.grad = g
                decayed.append(p)
            groups = [{"params": decayed, "weight_decay": weight_decay},
                      {"params": [self.flat.flat[False]], "weight_decay": 0.0}]
        else:
            groups = [{"params": [self.flat.flat[True]], "weight_decay": weight_decay},
                      {"params": [self.flat.flat[False]], "weight_decay": 0.0}]
        self.opt = torch.optim.AdamW(groups, lr=lr, betas=tuple(betas), eps=eps,
                                     fused=dev.type == "cuda")
        # in-place gathers of updated slices still in flight: bucket -> work
        self._gathers: Dict[int, object] = {}
        self._bucket_of = {n: bi for bi, (_, _, _, names) in enumerate(self._buckets) for n in names}
        if self._shard:
            self.flat.fence = self._fence
        self._pending: Dict[int, int] = {}
        self._hooks = []
        if self._buckets:
            owner = {}
            for bi, (_, _, _, names) in enumerate(self._buckets):
                for n in names:
                    owner[n] = bi
            for name, p in self.flat.params.items():
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad(owner[name])))

    # ------------------------------------------------------------ buckets
    def _make_buckets(self, bucket_bytes: int) -> List[Tuple[bool, int, int, List[str]]]:
        """Consecutive parameters of each flat buffer, grouped up to
        ``bucket_bytes`` (a parameter larger than that is a bucket alone)."""
        limit = max(1, bucket_bytes // 4)
        buckets = []
        for decay in (True, False):
            cur, start, end = [], None, None
            for sp in self.flat.specs:
                d, a, b = self.flat.slices[sp.name]
                if d != decay:
                    continue
                if cur and b - start > limit:
                    buckets.append((decay, start, end, cur))
                    cur = []
                if not cur:
                    start = a
                cur.append(sp.name)
                end = b
            if cur:
                buckets.append((decay, start, end, cur))
        return buckets

    def _on_grad(self, bi: int):
        def hook(_p):
            if not self._last:
                return
            left = self._pending.get(bi, len(self._buckets[bi][3])) - 1
            self._pending[bi] = left
            if left == 0:
                decay, a, b, _ = self._buckets[bi]
                if bi in self._shard:
                    self._works.append(dist.reduce_scatter_tensor(self._shard[bi][1], self.flat.grad[decay][a:b],
                                                                  group=self.group, async_op=True))
                else:
                    self._works.append(dist.all_reduce(self.flat.grad[decay][a:b], group=self.group, async_op=True))
        return hook

    def _fence(self, name: str) -> None:
        """Wait (on the device) for the gather of ``name``'s bucket, once."""
        if self._gathers:
            w = self._gathers.pop(self._bucket_of.get(name, -1), None)
            if w is not None:
                w.wait()

    def _wait_gathers(self) -> None:
        for w in self._gathers.values():
            w.wait()
        self._gathers = {}

    # ------------------------------------------------------------ step
    def step(self, tokens: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One optimizer step on this rank's (b, T) tokens and targets.

        Returns the mean objective over the global batch as a device tensor
        (no host synchronisation).
        """
        b = tokens.shape[0]
        m = min(self.micro_batch, b)
        if b % m:
            raise ValueError(f"rank batch {b} is not a multiple of the micro-batch {m}")
        n_micro = b // m
        self.flat.zero_grad()
        self._pending = {}
        self._works = []
        loss_sum = torch.zeros((), dtype=torch.float32, device=tokens.device)
        for i in range(n_micro):
            self._last = i == n_micro - 1
            obj, _ = self.model.loss(tokens[i * m:(i + 1) * m], targets[i * m:(i + 1) * m])
            (obj / n_micro).backward()
            loss_sum += obj.detach()
        self._last = False
        if self.world > 1:
            if len(self._works) != len(self._buckets):
                raise RuntimeError(f"{len(self._buckets) - len(self._works)} gradient buckets were not "
                                   "all-reduced: some parameters received no gradient")
            for w in self._works:
                w.wait()
            self._works = []
        if self._shard:
            # the loss and this rank's share of ||g||^2 in one all-reduce
            red = torch.stack([loss_sum, self._local_sq()])
            dist.all_reduce(red, group=self.group)
            loss_sum = red[0]
            self._apply_clip(red[1])
        else:
            if self.world > 1:
                dist.all_reduce(loss_sum, group=self.group)
            self._clip_and_scale()
        loss = loss_sum / (n_micro * self.world)
        if self.check_finite:
            # loss and gnorm are already reduced over the ranks, so every rank
            # takes the same decision and no collective is left unmatched
            ok = bool(torch.isfinite(loss) & torch.isfinite(self.last_gnorm))
            if not ok:
                raise FloatingPointError(f"non-finite loss {float(loss)} or gradient norm "
                                         f"{float(self.last_gnorm)}; the update was not applied")
        self._wait_gathers()  # a bucket no forward fetched since the last step
        if self._ref_opt is not None:
            self._ref_opt.step(self._opt_step)
        else:
            self.opt.step()
        self._opt_step += 1
        if self._shard:
            # every rank's updated slices back into the full masters, in the
            # order the next forward needs them (the reverse of the buckets')
            for bi in sorted(self._shard, reverse=True):
                self._gathers[bi] = dist.all_gather_into_tensor(self._gather_out[bi], self._shard[bi][0],
                                                                group=self.group, async_op=True)
        if hasattr(self.model, "weights_changed"):
            self.model.weights_changed()
        return loss

    def _clip_and_scale(self) -> None:
        grads = list(self.flat.grad.values())
        norms = torch.stack([torch.linalg.vector_norm(g) for g in grads])
        gnorm = torch.linalg.vector_norm(norms) / self.world
        scale = torch.clamp(self.clip / torch.clamp(gnorm, min=1e-12), max=1.0) / self.world
        torch._foreach_mul_(grads, scale)
        self.last_gnorm = gnorm

    def _sharded_grads(self):
        """(this rank's gradient slices, the replicated gradients)."""
        shard = [g for _, g in self._shard.values()]
        repl = [self.flat.grad[True][a:b] for bi, (d, a, b, _) in enumerate(self._buckets)
                if d and bi not in self._shard]
        repl.append(self.flat.grad[False])
        return shard, repl

    def _local_sq(self) -> torch.Tensor:
        """This rank's share of the squared global norm: its slices, plus the
        replicated gradients counted on rank 0 only."""
        shard, repl = self._sharded_grads()
        parts = [torch.linalg.vector_norm(g) for g in shard]
        if self.rank == 0:
            parts += [torch.linalg.vector_norm(g) for g in repl]
        return torch.sum(torch.stack(parts) ** 2)

    def _apply_clip(self, total_sq: torch.Tensor) -> None:
        shard, repl = self._sharded_grads()
        gnorm = torch.sqrt(total_sq) / self.world
        scale = torch.clamp(self.clip / torch.clamp(gnorm, min=1e-12), max=1.0) / self.world
        torch._foreach_mul_(shard + repl, scale)
        self.last_gnorm = gnorm

    def close(self) -> None:
        self._wait_gathers()
        if self.flat.fence == self._fence:
            self.flat.fence = None
        for h in self._hooks:
            h.remove()
        self._hooks = []


def main(argv=None) -> None:
    """``python -m algx.train --profile-steps N``: time N config-5 training
    steps on one GPU on synthetic token ids and print tok/s (the reference
    trainer's ``--profile-steps`` mode, train.py:96)."""
    import argparse
    import json

    from .model import AlgebraicLM, config_125m, config_algebraic_125m, parse_overrides, train_flops_per_token

    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--profile-steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--batch", type=int, default=64, help="sequences per optimizer step")
    ap.add_argument("--micro", type=int, default=8, help="sequences per micro-batch")
    ap.add_argument("--preset", choices=("standard", "algebraic"), default="standard",
                    help="standard: BASELINE config 5 (SwiGLU, RoPE, ce); algebraic: the reference's algebraic preset")
    ap.add_argument("--set", action="append", default=[], metavar="KEY=VALUE",
                    help="override an LMConfig field, typed by the field (repeatable)")
    ap.add_argument("--layers", type=int, default=None, help="override n_layers (same as --set n_layers=N)")
    ap.add_argument("--check-finite", action="store_true",
                    help="raise FloatingPointError on a non-finite loss or gradient norm (one host sync per step)")
    ap.add_argument("--optimizer", default="adamw", choices=("adamw", "muon_adamw", "cadamw", "hybrid_muon_cadamw"),
                    help="adamw: fused AdamW (BASELINE config 5); the others: the reference trainer's optimizers")
    ap.add_argument("--lr", type=float, default=2e-3)
    ap.add_argument("--total-steps", type=int, default=1000, help="cosine schedule length (reference optimizers)")
    ap.add_argument("--ns-precision", choices=("default", "highest"), default="default",
                    help="Muon's Newton-Schulz matmuls: default = bf16 operands, float32 accumulation (XLA's "
                         "DEFAULT float32 dot on TPU); highest = float32 operands")
    args = ap.parse_args(argv)
    over = parse_overrides(args.set)
    if args.layers is not None:
        over["n_layers"] = args.layers
    cfg = (config_125m if args.preset == "standard" else config_algebraic_125m)(**over)
    dev = torch.device("cuda", torch.cuda.current_device())
    model = AlgebraicLM(cfg, device=dev, seed=0)
    tr = DataParallelTrainer(model, lr=args.lr, micro_batch=args.micro, check_finite=args.check_finite,
                             optimizer=args.optimizer, total_steps=args.total_steps,
                             opt_kwargs=None if args.optimizer == "adamw" else {"precision": args.ns_precision})
    g = torch.Generator(device=dev).manual_seed(777)
    seq = torch.randint(0, cfg.vocab_size, (args.batch, cfg.seq_len + 1), device=dev, generator=g)
    tok, tgt = seq[:, :-1].contiguous(), seq[:, 1:].contiguous()
    for _ in range(args.warmup):
        tr.step(tok, tgt)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    losses = [tr.step(tok, tgt) for _ in range(args.profile_steps)]
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / max(args.profile_steps, 1)
    tokens = args.batch * cfg.seq_len
    print(json.dumps({"tok_per_s": tokens / (ms / 1e3), "ms_per_step": ms,
                      "tflops_6P": train_flops_per_token(cfg) * tokens / (ms / 1e3) / 1e12,
                      "loss": [float(x) for x in losses], "gnorm": float(tr.last_gnorm), "batch": args.batch,
                      "micro": args.micro, "layers": cfg.n_layers, "preset": args.preset,
                      "optimizer": args.optimizer,
                      "ns_precision": None if args.optimizer == "adamw" else args.ns_precision}))


if __name__ == "__main__":
    main()
