"""Rotary position tables for the fused QK-norm -> rotary -> attention prologue.

The tables are (T, head_dim / 2) fp32 pairs (cos, sin) as the reference's
model builds them (model.py:128-134): trigonometric RoPE (standard.py:16-21)
or the Cayley rotations on a geometric frequency grid (algebraic.py:124-169).
They are built once per sequence length (not a hot path) in float32 on any
device and passed to ``qknorm_flash_attention(..., rotary=(cos, sin))``.
"""

from __future__ import annotations

import math

import torch


def rope_table(head_dim: int, seq_len: int, base: float = 10000.0, device=None):
    """cos, sin of t * base^(-i / half), i < half, in float32 (standard.py:16-21)."""
    half = head_dim // 2
    theta = 1.0 / (torch.tensor(base, dtype=torch.float32, device=device)
                   ** (torch.arange(half, dtype=torch.float32, device=device) / half))
    angles = torch.arange(seq_len, dtype=torch.float32, device=device)[:, None] * theta[None, :]
    return torch.cos(angles), torch.sin(angles)


def cayley_powers(w: torch.Tensor, seq_len: int):
    """Rows ((1 + i w)^2 / (1 + w^2))^m, m < seq_len, per frequency w (algebraic.py:124-149).

    Position m's rotation is the product of the squared base rotations of its
    set bits; every squaring is renormalised to unit length, and so is the
    final product.
    """
    w = w.to(torch.float32)
    w2 = w * w
    c = (1.0 - w2) / (1.0 + w2)
    s = (2.0 * w) / (1.0 + w2)
    pos = torch.arange(seq_len, device=w.device)
    out_c = torch.ones((seq_len, w.shape[0]), dtype=torch.float32, device=w.device)
    out_s = torch.zeros((seq_len, w.shape[0]), dtype=torch.float32, device=w.device)
    bit = 0
    while (1 << bit) < seq_len:
        take = ((pos >> bit) & 1).bool()[:, None]
        out_c, out_s = (torch.where(take, out_c * c - out_s * s, out_c),
                        torch.where(take, out_c * s + out_s * c, out_s))
        c, s = c * c - s * s, 2.0 * c * s
        inv = torch.rsqrt(c * c + s * s)
        c, s = c * inv, s * inv
        bit += 1
    inv = torch.rsqrt(out_c * out_c + out_s * out_s)
    return out_c * inv, out_s * inv


def cayley_table_geometric(head_dim: int, seq_len: int, base: float = 10000.0, w0: float = 0.5,
                           fraction: float = 1.0, device=None):
    """Cayley tables on the grid w_k = w0 * base^(-k / half), the first
    ``fraction * half`` frequencies rotating, the rest fixed (algebraic.py:152-169).
    base^(1/half) is taken by log2(half) square roots, as the reference does."""
    half = head_dim // 2
    levels = int(round(math.log2(half)))
    if 1 << levels != half:
        raise ValueError("geometric Cayley grid needs head_dim/2 to be a power of two")
    r = float(base)
    for _ in range(levels):
        r = math.sqrt(r)
    ratio = 1.0 / r
    active = int(round(fraction * half))
    w = torch.tensor([w0 * ratio ** i if i < active else 0.0 for i in range(half)], dtype=torch.float32,
                     device=device)
    return cayley_powers(w, seq_len)
