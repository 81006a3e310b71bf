"""The reference trainer's optimizers on torch tensors (optimizers.py:1-248):
Muon on the 2-D weight matrices + AdamW on the rest (``muon_adamw``),
cautious AdamW everywhere (``cadamw``), and Muon + cautious AdamW
(``hybrid_muon_cadamw``), with the cosine learning-rate schedule.

The update rules are the reference's, element for element; the schedule and
the Adam bias corrections are computed in float32 as the reference computes
them. Parameters are addressed by name: the reference's routing rule
(``is_muon_param``, optimizers.py:68-89) reads the last path component, and a
weight the model stores fused (``w_qkv`` = [w_q | w_k | w_v], ``w_gu`` =
[w_g | w_u], column blocks) is updated block by block, so each reference
matrix gets its own Newton-Schulz orthogonalisation and its own cautious mask
mean.
"""

from __future__ import annotations

import math
from typing import Iterable, List, Optional, Tuple

import torch
import torch.distributed as dist

# Quintic Newton-Schulz coefficients of the Muon optimizer (optimizers.py:38)
NS_COEFFS = (3.4445, -4.7750, 2.0315)
NAMES = ("muon_adamw", "cadamw", "hybrid_muon_cadamw")


PRECISIONS = ("highest", "default")


def _matmul_ops(precision: str, like: torch.Tensor):
    """(round an operand, multiply rounded operands) for a matmul precision.

    ``highest``: operands and products in the working dtype. ``default``:
    operands rounded to bf16, products accumulated in float32, which is what
    XLA's DEFAULT precision computes for a float32 dot on the TPU the
    reference trains on; on a CUDA float32 tensor it runs on the bf16 tensor
    cores with a float32 output."""
    if precision == "highest":
        return (lambda t: t), torch.matmul
    if precision != "default":
        raise ValueError(f"unknown matmul precision {precision!r}; choices: {PRECISIONS}")
    if like.is_cuda and like.dtype == torch.float32:
        def mm(a, b):
            f = torch.bmm if a.ndim == 3 else torch.mm
            return f(a, b, out_dtype=torch.float32)
        return (lambda t: t.to(torch.bfloat16)), mm
    dt = like.dtype
    return (lambda t: t.to(torch.bfloat16).to(dt)), torch.matmul


def _ns_iterations_tensor_cores(X: torch.Tensor, steps: int) -> torch.Tensor:
    """The iterations of newton_schulz_5 at ``default`` precision on a CUDA
    float32 batch (count, m, n), m <= n: bf16 operands on the tensor cores,
    float32 products, with each linear combination folded into the product
    that feeds it (beta * C + alpha * A @ B in the GEMM epilogue):
    B = b A + c A^2, X <- a X + B X, and the refinement as
    X <- 1.5 X - 0.5 A X. The operands are rounded to bf16 as in the literal
    sequence; the result differs from it only at that rounding level, and it
    saves the separate element-wise passes over the stacks."""
    a, b, c = NS_COEFFS
    f32, bf16 = torch.float32, torch.bfloat16
    fma_mm = torch.ops.aten.baddbmm.dtype
    for _ in range(steps):
        x = X.to(bf16)
        A = torch.bmm(x, x.transpose(-2, -1), out_dtype=f32)
        a16 = A.to(bf16)
        B = fma_mm(A, a16, a16, f32, beta=b, alpha=c)
        X = fma_mm(X, B.to(bf16), x, f32, beta=a, alpha=1.0)
    for _ in range(2):
        x = X.to(bf16)
        A = torch.bmm(x, x.transpose(-2, -1), out_dtype=f32)
        X = fma_mm(X, A.to(bf16), x, f32, beta=1.5, alpha=-0.5)
    return X


def newton_schulz_5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7, precision: str = "highest") -> torch.Tensor:
    """Orthogonalise the trailing two dimensions of G (optimizers.py:27-65):
    Frobenius pre-normalisation, ``steps`` quintic iterations, two order-3
    Schulz refinements, then scaling by sqrt(max(1, M / N)). The Gram
    matrices are min(M, N) square (G is transposed first when M > N).
    Leading dimensions are a batch of independent matrices."""
    if G.ndim < 2:
        return G
    if G.ndim > 3:
        return newton_schulz_5(G.reshape(-1, *G.shape[-2:]), steps, eps, precision).reshape(G.shape)
    lo, mm = _matmul_ops(precision, G)
    a, b, c = NS_COEFFS
    M, N = G.shape[-2], G.shape[-1]
    transposed = M > N
    X = G.transpose(-2, -1) if transposed else G
    X = X / torch.sqrt(torch.sum(X * X, dim=(-2, -1), keepdim=True) + eps)
    if precision == "default" and X.is_cuda and X.dtype == torch.float32:
        X = _ns_iterations_tensor_cores(X if X.ndim == 3 else X.unsqueeze(0), steps).reshape(X.shape)
        if transposed:
            X = X.transpose(-2, -1)
        return X * math.sqrt(max(1.0, float(M) / float(N)))
    for _ in range(steps):
        x = lo(X)
        A = mm(x, x.transpose(-2, -1))
        a16 = lo(A)
        B = b * A + c * mm(a16, a16)
        X = a * X + mm(lo(B), x)
    eye = torch.eye(min(M, N), dtype=X.dtype, device=X.device)
    for _ in range(2):
        x = lo(X)
        A = mm(x, x.transpose(-2, -1))
        X = 0.5 * mm(lo(3.0 * eye - A), x)
    if transposed:
        X = X.transpose(-2, -1)
    return X * math.sqrt(max(1.0, float(M) / float(N)))


def is_muon_param(name: str, ndim: int) -> bool:
    """The reference's routing (optimizers.py:68-89) on the last name component."""
    key = name.split(".")[-1]
    if key == "embed":
        return False
    if key.startswith("w_"):
        return True
    if key.startswith("ln") or key.endswith("_gain") or key == "sink" or "bias" in key:
        return False
    return ndim >= 2


def cosine_schedule(peak_lr: float, total_steps: int, warmup_fraction: float, min_lr_ratio: float):
    """Linear warm-up then cosine decay to peak * min_lr_ratio (optimizers.py:92-115),
    in float32 like the reference."""
    f32 = torch.float32
    warm = float(warmup_fraction) if warmup_fraction >= 1 else max(1.0, float(round(warmup_fraction * total_steps)))
    floor = peak_lr * min_lr_ratio

    def lr(step: int) -> torch.Tensor:
        t = torch.tensor(float(step), dtype=f32) + 1.0
        warm_f = torch.clamp(t / warm, max=1.0)
        prog = torch.clamp((t - warm) / max(1.0, float(total_steps) - warm), 0.0, 1.0)
        cos = floor + (peak_lr - floor) * 0.5 * (1.0 + torch.cos(math.pi * prog))
        return torch.where(t < warm, peak_lr * warm_f, cos)

    return lr


def reference_blocks(name: str, param: torch.Tensor) -> List[Tuple[str, torch.Tensor]]:
    """The reference parameters a (possibly fused) model parameter holds, as views."""
    key = name.split(".")[-1]
    base = name[: len(name) - len(key)]
    if key == "w_qkv":
        d = param.shape[1] // 3
        return [(base + k, param[:, i * d:(i + 1) * d]) for i, k in enumerate(("w_q", "w_k", "w_v"))]
    if key == "w_gu":
        f = param.shape[1] // 2
        return [(base + k, param[:, i * f:(i + 1) * f]) for i, k in enumerate(("w_g", "w_u"))]
    return [(name, param)]


class _Group:
    """Reference parameters of one shape, dtype and routing, updated together:
    their values and gradients are gathered into one (count, *shape) stack
    per step, the optimizer state lives stacked, and every per-matrix
    quantity (the Newton-Schulz normalisation, the cautious mask's mean) is
    taken per row of the stack."""

    def __init__(self, shape, decayed: bool, muon: bool, like: torch.Tensor):
        self.shape, self.decayed, self.muon = tuple(shape), decayed, muon
        self.like = like
        self.params: List[torch.Tensor] = []
        self.grads: List[torch.Tensor] = []
        self.names: List[str] = []
        self.m = self.v = None

    def add(self, name: str, p: torch.Tensor, g: torch.Tensor) -> None:
        self.names.append(name)
        self.params.append(p)
        self.grads.append(g)

    def init_state(self, rank: int = 0, world: int = 1) -> None:
        """State for the rows this rank updates: all of them (world 1), or a
        contiguous share of ceil(n / world) rows, padded with zero rows so that
        every rank's share has the same size for the all-gather."""
        n = len(self.params)
        self.world = world
        self.chunk = n if world == 1 else -(-n // world)
        self.lo = min(n, rank * self.chunk) if world > 1 else 0
        self.hi = min(n, self.lo + self.chunk)
        self.m = torch.zeros((self.chunk,) + self.shape, dtype=self.like.dtype, device=self.like.device)
        self.v = None if self.muon else torch.zeros_like(self.m)

    def own_stack(self, tensors: List[torch.Tensor]) -> torch.Tensor:
        """This rank's rows of ``tensors`` stacked, zero rows after them up to
        the share size (zero rows update to zero: no division by zero)."""
        own = tensors[self.lo:self.hi]
        if len(own) == self.chunk:
            return torch.stack(own)
        out = torch.zeros((self.chunk,) + self.shape, dtype=self.like.dtype, device=self.like.device)
        if own:
            out[:len(own)] = torch.stack(own)
        return out


class ReferenceOptimizer:
    """One of the reference's optimizers over named parameters (with .grad).

    ``params``: (name, tensor, decayed) triples; the tensors are updated in
    place. ``step(step)`` applies the update for the 0-based step index, with
    the learning rates of the reference's schedules (optimizers.py:153-154).
    ``precision`` is the Newton-Schulz matmul precision (``highest`` or
    ``default``, see ``_matmul_ops``). ``shard``: the ranks of ``group`` (a
    torch.distributed process group whose ranks hold the same parameters and
    gradients) split every Muon stack of at least as many matrices as ranks,
    each orthogonalising a contiguous share, and all-gather the updated
    matrices; the other stacks are updated on every rank.
    """

    def __init__(self, name: str, params: Iterable[Tuple[str, torch.Tensor, bool]], lr: float,
                 weight_decay: float = 0.1, total_steps: int = 1000, warmup_fraction: float = 0.02,
                 min_lr_ratio: float = 0.1, b1: float = 0.9, b2: float = 0.95, adam_eps: float = 1e-8,
                 muon_lr: Optional[float] = None, muon_wd: Optional[float] = None, muon_momentum: float = 0.95,
                 muon_steps: int = 5, cautious_eps: float = 1e-3, precision: str = "highest",
                 shard: bool = False, group=None):
        name = name.lower().strip()
        if name not in NAMES:
            raise ValueError(f"Unknown optimizer: {name}. Choices: {NAMES}")
        if precision not in PRECISIONS:
            raise ValueError(f"unknown matmul precision {precision!r}; choices: {PRECISIONS}")
        self.name = name
        self.precision = precision
        self.wd = weight_decay
        self.muon_wd = weight_decay if muon_wd is None else muon_wd
        self.b1, self.b2, self.eps = b1, b2, adam_eps
        self.mu, self.ns_steps, self.cautious_eps = muon_momentum, muon_steps, cautious_eps
        self.adam_lr = cosine_schedule(lr, total_steps, warmup_fraction, min_lr_ratio)
        self.muon_lr = cosine_schedule(lr if muon_lr is None else muon_lr, total_steps, warmup_fraction,
                                       min_lr_ratio)
        groups = {}
        for pname, p, decayed in params:
            if p.grad is None:
                raise ValueError(f"parameter {pname} has no .grad buffer")
            for (bname, pv), (_, gv) in zip(reference_blocks(pname, p.data), reference_blocks(pname, p.grad)):
                muon = name != "cadamw" and is_muon_param(bname, pv.ndim)
                key = (tuple(pv.shape), bool(decayed), muon, pv.dtype, pv.device)
                if key not in groups:
                    groups[key] = _Group(pv.shape, bool(decayed), muon, pv)
                groups[key].add(bname, pv, gv)
        self.groups: List[_Group] = list(groups.values())
        self.pg = group
        world = dist.get_world_size(group) if shard and dist.is_available() and dist.is_initialized() else 1
        rank = dist.get_rank(group) if world > 1 else 0
        self.sharded_groups = 0
        for grp in self.groups:
            split = grp.muon and world > 1 and len(grp.params) >= world
            grp.init_state(rank, world if split else 1)
            self.sharded_groups += int(split)

    @torch.no_grad()
    def step(self, step: int) -> None:
        f32 = torch.float32
        # The schedule, bias corrections and decay factors are float32
        # arithmetic, as in the reference, done on the host; their exact
        # float32 values reach the device ops as Python scalars. (A 0-d host
        # tensor moved to the device would be a pageable copy, which can hold
        # the host until the stream drains and then expose every launch of the
        # update.)
        t = torch.tensor(float(step + 1), dtype=f32)
        c1 = float(1.0 - torch.tensor(self.b1, dtype=f32) ** t)
        c2 = float(1.0 - torch.tensor(self.b2, dtype=f32) ** t)
        lr_a_t, lr_m_t = self.adam_lr(step), self.muon_lr(step)
        lr_a, lr_m = float(lr_a_t), float(lr_m_t)
        decay_a, decay_m = float(1.0 - lr_a_t * self.wd), float(1.0 - lr_m_t * self.muon_wd)
        for grp in self.groups:
            dev = grp.m.device
            g = grp.own_stack(grp.grads)
            p = grp.own_stack(grp.params)
            m, v = grp.m, grp.v
            if grp.muon:
                m.mul_(self.mu).add_((1.0 - self.mu) * g)
                x = (1.0 - self.mu) * g + self.mu * m
                # a 1-D matrix passes through unchanged (optimizers.py:35-36)
                o = newton_schulz_5(x, steps=self.ns_steps, precision=self.precision) if len(grp.shape) >= 2 else x
                p = p * (decay_m if grp.decayed else 1.0) - lr_m * o
            else:
                m.mul_(self.b1).add_((1.0 - self.b1) * g)
                v.mul_(self.b2).add_((1.0 - self.b2) * (g * g))
                u = (m / c1) / (torch.sqrt(v / c2) + self.eps)
                if self.name != "muon_adamw":  # cautious: keep the components that agree with the gradient
                    # the reference's 0/1 mask is built from Python scalars: float32
                    mask = (u * g > 0.0).to(f32)
                    mean = mask.mean(dim=tuple(range(1, mask.ndim)), keepdim=True) if mask.ndim > 1 else mask
                    u = u * (mask / torch.clamp(mean, min=self.cautious_eps))
                p = p * (decay_a if grp.decayed else 1.0) - lr_a * u
            if grp.world > 1:
                full = torch.empty((grp.world * grp.chunk,) + grp.shape, dtype=p.dtype, device=dev)
                dist.all_gather_into_tensor(full, p.contiguous(), group=self.pg)
                p = full[:len(grp.params)]
            torch._foreach_copy_(grp.params, list(p.unbind(0)))
