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

# Quintic Newton-Schulz coefficients of the Muon optimizer (optimizers.py:38)
NS_COEFFS = (3.4445, -4.7750, 2.0315)
NAMES = ("muon_adamw", "cadamw", "hybrid_muon_cadamw")


def newton_schulz_5(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Orthogonalise the trailing two dimensions of G (optimizers.py:27-65):
    Frobenius pre-normalisation, ``steps`` quintic iterations, two order-3
    Schulz refinements, then scaling by sqrt(max(1, M / N)). The Gram
    matrices are min(M, N) square (G is transposed first when M > N)."""
    if G.ndim < 2:
        return G
    a, b, c = NS_COEFFS
    M, N = G.shape[-2], G.shape[-1]
    transposed = M > N
    X = G.transpose(-2, -1) if transposed else G
    X = X / torch.sqrt(torch.sum(X * X, dim=(-2, -1), keepdim=True) + eps)
    for _ in range(steps):
        A = X @ X.transpose(-2, -1)
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    eye = torch.eye(min(M, N), dtype=X.dtype, device=X.device)
    for _ in range(2):
        A = X @ X.transpose(-2, -1)
        X = 0.5 * ((3.0 * eye - A) @ X)
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


class ReferenceOptimizer:
    """One of the reference's optimizers over named parameters (with .grad).

    ``params``: (name, tensor, decayed) triples; the tensors are updated in
    place. ``step(step)`` applies the update for the 0-based step index, with
    the learning rates of the reference's schedules (optimizers.py:153-154).
    """

    def __init__(self, name: str, params: Iterable[Tuple[str, torch.Tensor, bool]], lr: float,
                 weight_decay: float = 0.1, total_steps: int = 1000, warmup_fraction: float = 0.02,
                 min_lr_ratio: float = 0.1, b1: float = 0.9, b2: float = 0.95, adam_eps: float = 1e-8,
                 muon_lr: Optional[float] = None, muon_wd: Optional[float] = None, muon_momentum: float = 0.95,
                 muon_steps: int = 5, cautious_eps: float = 1e-3):
        name = name.lower().strip()
        if name not in NAMES:
            raise ValueError(f"Unknown optimizer: {name}. Choices: {NAMES}")
        self.name = name
        self.wd = weight_decay
        self.muon_wd = weight_decay if muon_wd is None else muon_wd
        self.b1, self.b2, self.eps = b1, b2, adam_eps
        self.mu, self.ns_steps, self.cautious_eps = muon_momentum, muon_steps, cautious_eps
        self.adam_lr = cosine_schedule(lr, total_steps, warmup_fraction, min_lr_ratio)
        self.muon_lr = cosine_schedule(lr if muon_lr is None else muon_lr, total_steps, warmup_fraction,
                                       min_lr_ratio)
        self.slots = []  # (name, param view, grad view, decayed, uses Muon, m, v)
        for pname, p, decayed in params:
            if p.grad is None:
                raise ValueError(f"parameter {pname} has no .grad buffer")
            for (bname, pv), (_, gv) in zip(reference_blocks(pname, p.data), reference_blocks(pname, p.grad)):
                muon = name != "cadamw" and is_muon_param(bname, pv.ndim)
                m = torch.zeros_like(pv, memory_format=torch.contiguous_format)
                v = None if muon else torch.zeros_like(pv, memory_format=torch.contiguous_format)
                self.slots.append((bname, pv, gv, bool(decayed), muon, m, v))

    @torch.no_grad()
    def step(self, step: int) -> None:
        f32 = torch.float32
        t = torch.tensor(float(step + 1), dtype=f32)
        c1 = 1.0 - torch.tensor(self.b1, dtype=f32) ** t
        c2 = 1.0 - torch.tensor(self.b2, dtype=f32) ** t
        lr_a, lr_m = self.adam_lr(step), self.muon_lr(step)
        for _, p, g, decayed, muon, m, v in self.slots:
            dev = p.device
            if muon:
                m.mul_(self.mu).add_((1.0 - self.mu) * g)
                o = newton_schulz_5((1.0 - self.mu) * g + self.mu * m, steps=self.ns_steps)
                lr = lr_m.to(dev)
                decay = (1.0 - lr * self.muon_wd) if decayed else torch.ones((), dtype=f32, device=dev)
                p.copy_(p * decay - lr * o)
                continue
            m.mul_(self.b1).add_((1.0 - self.b1) * g)
            v.mul_(self.b2).add_((1.0 - self.b2) * (g * g))
            u = (m / c1.to(dev)) / (torch.sqrt(v / c2.to(dev)) + self.eps)
            if self.name != "muon_adamw":  # cautious: keep the components that agree with the gradient
                # the reference's 0/1 mask is built from Python scalars: float32
                mask = (u * g > 0.0).to(f32)
                u = u * (mask / torch.clamp(mask.mean(), min=self.cautious_eps))
            lr = lr_a.to(dev)
            decay = (1.0 - lr * self.wd) if decayed else torch.ones((), dtype=f32, device=dev)
            p.copy_(p * decay - lr * u)
