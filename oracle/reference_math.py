"""CPU restatement of the reference maths (torch-CPU, float64 by default).

TEST INFRASTRUCTURE ONLY. This module is the parity oracle for the CUDA
kernels in ``algebraic-extra_b200/``. It restates, function by function, the
dense maths of ``tasmaikeni13/algebraic-extra`` (paths below are relative to
that project) and the kernel-level semantics its Pallas kernels add (clamps,
row statistics, sink VJP, range guard, vocabulary label compare).

Gradients come from torch autograd on the dense float64 formulas. That is an
independent check of the kernels' hand-written VJPs, exactly as the reference
tests check its Pallas VJPs against JAX autodiff of the dense path.

Rounding points. The reference casts to the I/O dtype at a few places
(``p.astype(v.dtype)`` before P.V, ``out.astype(q.dtype)``, ``y.astype(x.dtype)``
in RMS norm, ``q_scaled`` in the flash wrapper, ``dz`` to ``h.dtype`` in the
fused head). Every oracle function takes the I/O dtype and applies the same
casts (a straight-through round trip in autograd), so a bfloat16 run of the
oracle reproduces the reference's rounding points while the arithmetic in
between stays float64.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own
``algebraic.py`` / ``standard.py`` / ``evaluation.py`` source and stores the
outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this
module against them, and ``tests/test_oracle_identities.py`` ports the
reference's closed-form identities (``tests/test_components.py``).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

F64 = torch.float64


# ---------------------------------------------------------------------------
# scalar helpers
# ---------------------------------------------------------------------------

def _round(x: torch.Tensor, dtype: Optional[torch.dtype]) -> torch.Tensor:
    """Round ``x`` through ``dtype`` and back (identity for None/float64)."""
    if dtype is None or dtype == x.dtype or dtype == F64:
        return x
    return x.to(dtype).to(x.dtype)


def rho(x: torch.Tensor) -> torch.Tensor:
    """x + sqrt(1+x^2) without cancellation for x<0 (algebraic.py:31-35)."""
    rad = 1.0 + x * x
    t = torch.abs(x) + rad * torch.rsqrt(rad)
    return torch.where(x >= 0, t, 1.0 / t)


def rho_exact(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(rho(x), 1/sqrt(1+x^2)) in the stable form (kernels/flash.py:76-80)."""
    rad = 1.0 + x * x
    r = torch.rsqrt(rad)
    t = torch.abs(x) + rad * r
    return torch.where(x >= 0, t, 1.0 / t), r


def rho_fast(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """(x + rad*rsqrt(rad), rsqrt(rad)) without the reciprocal (kernels/flash.py:83-88)."""
    rad = 1.0 + x * x
    r = torch.rsqrt(rad)
    return x + rad * r, r


def int_pow(x, n: int):
    """x**n by binary exponentiation (algebraic.py:38-51, kernels/flash.py:95-104)."""
    n = int(n)
    if n < 1:
        raise ValueError("n must be a positive integer")
    result = None
    base = x
    while n:
        if n & 1:
            result = base if result is None else result * base
        n >>= 1
        if n:
            base = base * base
    return result


def inv_root(l: torch.Tensor, n: int) -> torch.Tensor:
    """l^(-1/n) for n a power of two by rsqrt chains (kernels/flash.py:107-114)."""
    y = torch.rsqrt(l)
    k = n // 2
    while k > 1:
        y = y * torch.rsqrt(y)
        k //= 2
    return y


def root(value: float, n: int) -> float:
    """value^(1/n) for n a power of two by repeated sqrt (kernels/flash.py:117-123)."""
    out = float(value)
    while n > 1:
        out = math.sqrt(out)
        n //= 2
    return out


def attention_clamp(seq_len: int, n: int) -> float:
    """Upper score clamp of the unshifted asinh kernel (kernels/flash.py:747-748)."""
    t = root(1e37 / (seq_len + 1), n)
    return 0.5 * (t - 1.0 / t)


def likelihood_clamp(vocab: int, n: int) -> float:
    """Kernel-argument clamp of the algebraic head (algebraic.py:277-283, fused_head.py:273)."""
    out = 1e38 / vocab
    k = n
    while k > 1:
        out = math.sqrt(out)
        k //= 2
    return 0.25 * out


def kernel_sink_logit(omega: float, n: int, c: float) -> float:
    """Sink logit b with rho(b/c)^n = omega (algebraic.py:54-69)."""
    if omega <= 0:
        raise ValueError("omega must be positive")
    t = float(omega)
    k = int(round(math.log2(n)))
    if 1 << k != n:
        raise ValueError("n must be a power of two")
    for _ in range(k):
        t = math.sqrt(t)
    return c * 0.5 * (t - 1.0 / t)


# ---------------------------------------------------------------------------
# RMS / QK norm
# ---------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, gain: Optional[torch.Tensor], eps: float = 1e-5,
             io_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """RMS norm (algebraic.py:76-83); ``io_dtype`` reproduces ``y.astype(x.dtype)``.

    ``x`` arrives in float64 holding values representable in ``io_dtype``.
    The QK-norm kernel API (kernels/qk_norm.py:62-76) computes exactly this
    in the forward and JAX AD of it in the backward.
    """
    tau = torch.rsqrt(torch.mean(x * x, dim=-1, keepdim=True) + eps)
    y = x * tau
    if gain is not None:
        y = y * gain
    return _round(y, io_dtype)


class _Alu(torch.autograd.Function):
    """alu with the reference's own VJP rule (algebraic.py:104-113)."""

    @staticmethod
    def forward(ctx, x, beta, io_dtype):
        bz = beta * x
        r = torch.rsqrt(1.0 + bz * bz)
        u = bz * r
        one_plus_u = torch.where(bz < 0, (r * r) / (1.0 - u), 1.0 + u)
        ctx.save_for_backward(u, r)
        ctx.io = io_dtype
        return _round(0.5 * x * one_plus_u, io_dtype)

    @staticmethod
    def backward(ctx, g):
        u, r = ctx.saved_tensors
        derivative = 0.5 * (1.0 + u) + 0.5 * u * (r * r)
        return _round(g * derivative, ctx.io), None, None


def alu(x: torch.Tensor, beta: float = 1.0, io_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Algebraic linear unit x/2 (1 + bx / sqrt(1 + b^2 x^2)) (algebraic.py:86-101):
    for bx < 0 the factor 1 + u is r^2 / (1 - u); the result is rounded to
    ``io_dtype`` (``.astype(x.dtype)``), and so is the gradient."""
    return _Alu.apply(x, float(beta), io_dtype)


def qk_norm_backward(x: torch.Tensor, gain: torch.Tensor, dy: torch.Tensor, eps: float):
    """(dx, dgain) of ``rms_norm`` by autograd (kernels/qk_norm.py:41-55)."""
    xx = x.detach().clone().requires_grad_(True)
    gg = gain.detach().clone().requires_grad_(True)
    y = rms_norm(xx, gg, eps)
    y.backward(dy)
    return xx.grad, gg.grad


# ---------------------------------------------------------------------------
# rotary position tables (model.py:128-134) and the rotation (model.py:173-174)
# ---------------------------------------------------------------------------

def rope_table(head_dim: int, seq_len: int, base: float = 10000.0, dtype=torch.float32):
    """Trigonometric RoPE tables (standard.py:16-21): theta_i = base^(-i/half),
    angle = t * theta_i, all in ``dtype`` (the reference uses float32)."""
    half = head_dim // 2
    theta = 1.0 / (torch.tensor(base, dtype=dtype) ** (torch.arange(half, dtype=dtype) / half))
    angles = torch.arange(seq_len, dtype=dtype)[:, None] * theta[None, :]
    return torch.cos(angles), torch.sin(angles)


def cayley_powers(w: torch.Tensor, seq_len: int):
    """Rows ((1 + i w)^2 / (1 + w^2))^m for m < seq_len (algebraic.py:124-149):
    binary exponentiation over the bits of m with a renormalised squaring per
    bit, then a final renormalisation; in the dtype of ``w``."""
    w2 = w * w
    c = (1.0 - w2) / (1.0 + w2)
    s = (2.0 * w) / (1.0 + w2)
    positions = torch.arange(seq_len)
    out_c = torch.ones((seq_len, w.shape[0]), dtype=w.dtype)
    out_s = torch.zeros((seq_len, w.shape[0]), dtype=w.dtype)
    bit = 0
    while (1 << bit) < seq_len:
        take = ((positions >> bit) & 1).bool()[:, None]
        new_c = out_c * c - out_s * s
        new_s = out_c * s + out_s * c
        out_c = torch.where(take, new_c, out_c)
        out_s = torch.where(take, new_s, out_s)
        c, s = c * c - s * s, 2.0 * c * s
        inv = torch.rsqrt(c * c + s * s)
        c, s = c * inv, s * inv
        bit += 1
    inv = torch.rsqrt(out_c * out_c + out_s * out_s)
    return out_c * inv, out_s * inv


def cayley_table_geometric(head_dim: int, seq_len: int, base: float = 10000.0, w0: float = 0.5,
                           fraction: float = 1.0, dtype=torch.float32):
    """Geometric Cayley grid w_k = w0 * base^(-k/half) (algebraic.py:152-169)."""
    half = head_dim // 2
    levels = int(round(math.log2(half)))
    if 1 << levels != half:
        raise ValueError("geometric Cayley grid needs head_dim/2 to be a power of two")
    ratio = 1.0 / root(base, half)
    active = int(round(fraction * half))
    w = torch.tensor([w0 * ratio ** i if i < active else 0.0 for i in range(half)], dtype=dtype)
    return cayley_powers(w, seq_len)


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 io_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Rotate-half rotation of (..., T, D) by (>= T, D/2) tables (algebraic.py:172-179).

    With ``io_dtype`` the tables are first rounded to it (``cos.astype(x.dtype)``)
    and the rotated value is rounded to it once, the arithmetic in between
    staying in x's (wider) dtype.
    """
    half = x.shape[-1] // 2
    t = x.shape[-2]
    c = _round(cos[:t].to(x.dtype), io_dtype)
    s = _round(sin[:t].to(x.dtype), io_dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return _round(torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1), io_dtype)


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------

def _causal(t: int) -> torch.Tensor:
    return torch.tril(torch.ones((t, t), dtype=torch.bool))


def asinh_power_weights(scores, mask, n: int, c: float, sink_logit=None):
    """Normalised rho(s/c)^n with max shift and optional sink (algebraic.py:186-204)."""
    x = scores / c
    m = torch.amax(torch.where(mask, x, torch.full_like(x, -1e30)), dim=-1, keepdim=True)
    xb = None
    if sink_logit is not None:
        xb = sink_logit / c
        m = torch.maximum(m, xb)
    m = m.detach()
    shift = rho(-m)
    w = torch.where(mask, int_pow(rho(x) * shift, n), torch.zeros_like(x))
    denom = torch.sum(w, dim=-1, keepdim=True)
    if xb is not None:
        denom = denom + int_pow(rho(xb) * shift, n)
    return w / denom


def asinh_attention(q, k, v, *, n: int, c: float, sink_logit=None,
                    io_dtype: Optional[torch.dtype] = None):
    """Dense causal asinh-power attention on (B,H,T,D) (algebraic.py:207-216)."""
    d = q.shape[-1]
    t = q.shape[-2]
    scores = torch.einsum("bhqd,bhkd->bhqk", q, k) * (1.0 / math.sqrt(d))
    mask = _causal(t)[None, None]
    p = asinh_power_weights(scores, mask, n, c, sink_logit)
    out = torch.einsum("bhqk,bhkd->bhqd", _round(p, io_dtype), v)
    return _round(out, io_dtype)


def softmax_attention(q, k, v, *, sink_logit=None, io_dtype: Optional[torch.dtype] = None):
    """Dense causal softmax attention with optional sink (standard.py:24-38)."""
    d = q.shape[-1]
    t = q.shape[-2]
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) * (1.0 / math.sqrt(d))
    mask = _causal(t)[None, None]
    s = torch.where(mask, s, torch.full_like(s, -1e30))
    if sink_logit is not None:
        b = torch.broadcast_to(sink_logit, s.shape[:-1] + (1,))
        p = torch.softmax(torch.cat([s, b], dim=-1), dim=-1)[..., :-1]
    else:
        p = torch.softmax(s, dim=-1)
    out = torch.einsum("bhqk,bhkd->bhqd", _round(p, io_dtype), v)
    return _round(out, io_dtype)


def resolve_variant(kind: str, n: int, c: float, seq_len: int, shift=None, fast_rho=None,
                    inv_stat=None, range_guard: bool = False) -> dict:
    """Variant flags of the public wrapper (kernels/flash.py:732-760, 834-852).

    Returns a dict with ``mode`` in {"softmax", "clipped", "shifted", "guarded"}.
    """
    if kind == "softmax":
        return {"mode": "softmax"}
    if kind != "asinh":
        raise ValueError(f"unknown attention kernel: {kind}")
    if n < 2 or n & (n - 1):
        raise ValueError("asinh kernel needs n to be a power of two")
    if not math.isfinite(c) or c <= 0:
        raise ValueError("asinh scale c must be positive and finite")
    clamp = attention_clamp(seq_len, n)
    if shift is None:
        shift = clamp < 20.0
    if fast_rho is None:
        fast_rho = True
    if inv_stat is None:
        inv_stat = not shift
    if inv_stat and shift:
        raise ValueError("inverse-denominator statistic requires shift=False")
    guarded = bool(range_guard) and n <= 32
    mode = "guarded" if guarded else ("shifted" if shift else "clipped")
    return {"mode": mode, "clamp": clamp, "shift": bool(shift), "fast_rho": bool(fast_rho),
            "inv_stat": bool(inv_stat)}


def guard_in_range(q_scaled, k, v, sink_kernel: Optional[torch.Tensor], seq_len: int,
                   n: int, clamp: float) -> bool:
    """Range-guard decision of kernels/flash.py:840-849 (kernel units)."""
    bound = min(16.0, clamp / 2)
    q2 = float(torch.max(torch.sum(q_scaled.double() ** 2, dim=-1)))
    k2 = float(torch.max(torch.sum(k.double() ** 2, dim=-1)))
    ok = q2 * k2 <= (bound / 1.01) ** 2
    has_sink = sink_kernel is not None
    if has_sink:
        ok = ok and float(torch.max(torch.abs(sink_kernel.double()))) <= bound / 1.01
    vmax = min(1e8, 1e37 / ((seq_len + int(has_sink)) * (2 * bound + 1) ** n))
    ok = ok and float(torch.max(torch.abs(v.double()))) <= vmax
    return bool(ok)


def flash_attention(q, k, v, sink_logit=None, *, kind: str = "softmax", n: int = 16,
                    c: float = 16.0, shift=None, fast_rho=None, inv_stat=None,
                    range_guard: bool = False, io_dtype: Optional[torch.dtype] = None):
    """The function the reference's ``flash_attention`` evaluates (kernels/flash.py:763-857).

    Inputs are float64 tensors holding ``io_dtype`` values. The scale fold
    ``q_scaled = (q*scale).astype(q.dtype)`` (flash.py:823-833) is applied
    with the same rounding. The "clipped" variant (explicit ``shift=False``
    without the guard) evaluates ``rho(min(x, clamp))^n`` with a zero VJP at
    and above the clamp (flash.py:228, 357-360, 698-704); every other variant
    evaluates the dense function of algebraic.py:186-216 (the guarded low
    and high branches and the explicit shifted branch differ only in
    rounding). ``sink_logit`` is broadcastable to (H,).
    """
    B, H, T, D = q.shape
    var = resolve_variant(kind, n, c, T, shift, fast_rho, inv_stat, range_guard)
    unit = 1.0 if kind == "softmax" else float(c)
    scale = 1.0 / (math.sqrt(D) * unit)
    sink = None
    if sink_logit is not None:
        sink = torch.broadcast_to(torch.reshape(sink_logit, (-1,)), (H,)) / unit
    q_scaled = _round(q * scale, io_dtype)
    s = torch.einsum("bhqd,bhkd->bhqk", q_scaled, k)          # kernel units
    mask = _causal(T)[None, None]
    if var["mode"] == "softmax":
        s = torch.where(mask, s, torch.full_like(s, -1e30))
        if sink is not None:
            b = torch.broadcast_to(sink[None, :, None, None], s.shape[:-1] + (1,))
            p = torch.softmax(torch.cat([s, b], dim=-1), dim=-1)[..., :-1]
        else:
            p = torch.softmax(s, dim=-1)
    elif var["mode"] == "clipped":
        cl = var["clamp"]
        x = torch.where(s < cl, s, torch.full_like(s, cl))
        w = torch.where(mask, int_pow(rho(x), n), torch.zeros_like(x))
        denom = torch.sum(w, dim=-1, keepdim=True)
        if sink is not None:
            b = torch.where(sink < cl, sink, torch.full_like(sink, cl))
            denom = denom + int_pow(rho(b), n)[None, :, None, None]
        p = w / denom
    else:
        p = asinh_power_weights(s, mask, n, 1.0,
                                None if sink is None else sink[None, :, None, None])
    out = torch.einsum("bhqk,bhkd->bhqd", _round(p, io_dtype), v)
    return _round(out, io_dtype)


def attention_grads(fn, q, k, v, g, sink=None):
    """Autograd VJP of ``fn(q,k,v,sink)`` against cotangent ``g``; returns (o, dq, dk, dv, dsink)."""
    leaves = [t.detach().clone().requires_grad_(True) for t in (q, k, v)]
    s_leaf = None if sink is None else sink.detach().clone().requires_grad_(True)
    o = fn(*leaves, s_leaf)
    torch.sum(o * g).backward()
    return (o.detach(), leaves[0].grad, leaves[1].grad, leaves[2].grad,
            None if s_leaf is None else s_leaf.grad)


def sink_mass_and_slope(sink_kernel, stat, n: int, clamp: float, *, clipped: bool,
                        inv_stat: bool):
    """Per-row sink mass and d(logit)/d(sink) (kernels/flash.py:694-705)."""
    b = torch.minimum(sink_kernel, torch.full_like(sink_kernel, clamp)) if clipped else sink_kernel
    rb, r = rho_exact(b)
    if inv_stat:
        mass = int_pow(rb[None, :, None], n) * stat
    else:
        mass = int_pow(rb[None, :, None] * stat, n)
    slope = n * r
    if clipped:
        slope = torch.where(sink_kernel < clamp, slope, torch.zeros_like(slope))
    return mass, slope


# ---------------------------------------------------------------------------
# training heads on materialised logits
# ---------------------------------------------------------------------------

def algebraic_probs(z, n: int, c: float):
    """p_j ~ rho(z_j/c)^n, max shifted (algebraic.py:223-228)."""
    x = z / c
    m = torch.amax(x, dim=-1, keepdim=True).detach()
    w = int_pow(rho(x) * rho(-m), n)
    return w / torch.sum(w, dim=-1, keepdim=True)


def _gather_wrapped(p, targets):
    """take_along_axis with NumPy/JAX negative-index normalisation (algebraic.py:244)."""
    idx = torch.where(targets < 0, targets + p.shape[-1], targets).long()
    return torch.gather(p, -1, idx[:, None])[:, 0]


def algebraic_likelihood(z, targets, n: int, c: float):
    """(mean(1-p_t), p_t) forward of algebraic.py:231-245."""
    p = algebraic_probs(z, n, c)
    pt = _gather_wrapped(p, targets)
    return torch.mean(1.0 - pt), pt


def algebraic_likelihood_grad(z, targets, n: int, c: float, g_obj: float = 1.0):
    """Custom VJP of algebraic.py:255-262: (g n/c/N) r (p - y)."""
    p = algebraic_probs(z, n, c)
    x = z / c
    r = torch.rsqrt(1.0 + x * x)
    y = (torch.arange(p.shape[-1])[None, :] == targets[:, None]).to(p.dtype)
    return (g_obj * (n / c) / p.shape[0]) * r * (p - y)


def algebraic_likelihood_lean(z, targets, n: int, c: float):
    """Lean forward (algebraic.py:286-301)."""
    x = torch.minimum(z / c, torch.full_like(z, likelihood_clamp(z.shape[-1], n)))
    rad = 1.0 + x * x
    w = int_pow(x + rad * torch.rsqrt(rad), n)
    wt = _gather_wrapped(w, targets)
    pt = wt / torch.sum(w, dim=-1)
    return torch.mean(1.0 - pt), pt


def cross_entropy(z, targets):
    """(mean NLL, per-token NLL) of standard.py:41-47."""
    lse = torch.logsumexp(z, dim=-1)
    zt = _gather_wrapped(z, targets)
    nll = lse - zt
    return torch.mean(nll), nll.detach()


def logprob_from_logits(z, targets, head: str = "alg_ce", n: int = 8, c: float = 2.0):
    """Per-token log p(target) (evaluation.py:13-23)."""
    if head == "ce":
        a = z
    elif head == "alg_ce":
        a = n * torch.asinh(z / c)
    else:
        raise ValueError(f"unknown head {head!r}")
    return _gather_wrapped(torch.log_softmax(a, dim=-1), targets)


# ---------------------------------------------------------------------------
# fused LM head: the function kernels/fused_head.py evaluates
# ---------------------------------------------------------------------------

def fused_head_forward(h, embed, targets, *, kind: str = "ce", n: int = 16, c: float = 16.0,
                       ignore_index: Optional[int] = None,
                       io_dtype: Optional[torch.dtype] = None):
    """(objective, telemetry, stat, zt) of kernels/fused_head.py:72-117, 219-229, 260-275.

    The label compare is ``col == target`` (fused_head.py:86-87): a label
    outside [0, V) matches no column, so its target logit is 0 and its row
    still counts in the mean. ``ignore_index`` (an extension, default None =
    the reference) drops rows equal to it from the objective, the gradients
    and the mean; their telemetry is 0.
    """
    e = _round(embed, io_dtype)                    # embed.astype(h.dtype), fused_head.py:168
    z = h @ e.T
    N, V = z.shape
    cols = torch.arange(V)[None, :]
    onehot = (cols == targets[:, None]).to(z.dtype)
    zt = torch.sum(onehot * z, dim=-1)
    valid = torch.ones(N, dtype=torch.bool) if ignore_index is None else targets != ignore_index
    if kind == "ce":
        stat = torch.logsumexp(z, dim=-1)
        tel = stat - zt
    elif kind == "alg_ce":
        X = likelihood_clamp(V, n)
        x = torch.minimum(z / c, torch.full_like(z, X))
        rad = 1.0 + x * x
        w = int_pow(x + rad * torch.rsqrt(rad), n)
        stat = inv_root(torch.sum(w, dim=-1), n)
        xt = torch.minimum(zt / c, torch.full_like(zt, X))
        rt, _ = rho_exact(xt)
        tel = int_pow(rt * stat, n)
    else:
        raise ValueError(kind)
    tel = torch.where(valid, tel, torch.zeros_like(tel))
    count = max(int(valid.sum()), 1) if ignore_index is not None else N
    if kind == "ce":
        obj = torch.sum(tel) / count
    else:
        obj = torch.sum(torch.where(valid, 1.0 - tel, torch.zeros_like(tel))) / count
    return obj, tel, stat, zt


def fused_head_backward(h, embed, targets, *, kind: str = "ce", n: int = 16, c: float = 16.0,
                        g_obj: float = 1.0, ignore_index: Optional[int] = None,
                        io_dtype: Optional[torch.dtype] = None):
    """(dh, dembed) of kernels/fused_head.py:120-156, 194-216, 247-254.

    dz = softmax(z) - y (ce) or (p - y) r (alg_ce), masked for ignored rows,
    scaled by g*slope/count and rounded to ``io_dtype`` (``dzb``), then
    dh = dzb E and dE = dzb^T h.
    """
    _, _, stat, _ = fused_head_forward(h, embed, targets, kind=kind, n=n, c=c,
                                       ignore_index=ignore_index, io_dtype=io_dtype)
    e = _round(embed, io_dtype)
    z = h @ e.T
    N, V = z.shape
    cols = torch.arange(V)[None, :]
    y = (cols == targets[:, None]).to(z.dtype)
    valid = torch.ones(N, dtype=torch.bool) if ignore_index is None else targets != ignore_index
    count = max(int(valid.sum()), 1) if ignore_index is not None else N
    if kind == "ce":
        dz = torch.exp(z - stat[:, None]) - y
        slope = 1.0
    else:
        X = likelihood_clamp(V, n)
        x = torch.minimum(z / c, torch.full_like(z, X))
        rad = 1.0 + x * x
        r = torch.rsqrt(rad)
        p = int_pow((x + rad * r) * stat[:, None], n)
        dz = (p - y) * r
        slope = n / c
    dz = torch.where(valid[:, None], dz, torch.zeros_like(dz))
    dzb = _round(dz * (g_obj * slope / count), io_dtype)
    dh = _round(dzb @ e, io_dtype)
    de = dzb.T @ h
    return dh, de
