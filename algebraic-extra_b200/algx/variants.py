"""Variant resolution and kernel constants, in plain Python (no torch, no jax).

Shared by the torch front-end (``algx.kernels``) and the JAX front-end
(``algx_jax``), so both resolve the reference's options into the same C ABI
configuration and raise the same ``ValueError``s:

* attention: ``make_variant`` (kernels/flash.py:732-760), the option checks of
  ``flash_attention`` (kernels/flash.py:793-822) and the wrapper constants
  (scale fold, sink unit, range-guard bounds, kernels/flash.py:823-856);
* fused head: the objective constants (kernels/fused_head.py:260-275).
"""

from __future__ import annotations

import math
from typing import Optional

# C ABI enumerations (include/algx.h)
ALGX_F32, ALGX_BF16 = 0, 1
ALGX_ATTN_ASINH, ALGX_ATTN_SOFTMAX = 0, 1
ALGX_MODE_CLIPPED, ALGX_MODE_SHIFTED, ALGX_MODE_GUARDED = 0, 1, 2
ALGX_HEAD_CE, ALGX_HEAD_ALG_CE = 0, 1


def _root(value: float, n: int) -> float:
    """value^(1/n) for n a power of two by repeated sqrt (kernels/flash.py:117-123)."""
    out = float(value)
    while n > 1:
        out = math.sqrt(out)
        n //= 2
    return out


class Variant(dict):
    """Resolved asinh/softmax variant (mirrors kernels/flash.py:59-73)."""


def make_variant(kind: str, n: int = 16, c: float = 16.0, seq_len: int = 2048,
                 shift: Optional[bool] = None, fast_rho: Optional[bool] = None,
                 inv_stat: Optional[bool] = None, compact_stat: bool = True,
                 poly_rho: bool = False) -> Variant:
    """Variant resolution of kernels/flash.py:732-760."""
    if kind == "softmax":
        return Variant(kind="softmax", n=16, shift=True, fast_rho=False, clamp=0.0, inv_stat=False,
                       compact_stat=bool(compact_stat), poly_rho=False)
    if kind != "asinh":
        raise ValueError(f"unknown attention kernel: {kind}")
    if n < 2 or n & (n - 1):
        raise ValueError("asinh kernel needs n to be a power of two")
    if not math.isfinite(c) or c <= 0:
        raise ValueError("asinh scale c must be positive and finite")
    t = _root(1e37 / (seq_len + 1), n)
    clamp = 0.5 * (t - 1.0 / t)
    if shift is None:
        shift = clamp < 20.0
    if fast_rho is None:
        fast_rho = True
    if inv_stat is None:
        inv_stat = not shift
    if inv_stat and shift:
        raise ValueError("inverse-denominator statistic requires shift=False")
    if poly_rho and (shift or n != 16):
        raise ValueError("bounded radical approximation requires shift=False and n=16")
    return Variant(kind="asinh", n=int(n), shift=bool(shift), fast_rho=bool(fast_rho), clamp=float(clamp),
                   inv_stat=bool(inv_stat), compact_stat=bool(compact_stat), poly_rho=bool(poly_rho))


def check_flash_options(T: int, D: int, io_is_bf16: bool, *, kind: str, n: int, c: float, block: int,
                        block_q: Optional[int], block_k: Optional[int], shift, fast_rho, inv_stat,
                        compact_stat: bool, poly_rho: bool, range_guard: bool, resident_bwd, diagonal_bwd,
                        head_resident) -> Variant:
    """The option checks of ``flash_attention`` (kernels/flash.py:793-822) with the
    reference's error texts; returns the resolved variant. The schedule knobs are
    validated and otherwise ignored (the sm_100a kernels pick their own tiles)."""
    bq = min(block_q or block, T)
    bk = min(block_k or block, T)
    if T % bq or T % bk:
        raise ValueError(f"sequence length {T} must be divisible by blocks ({bq}, {bk})")
    var = make_variant(kind, n, c, T, shift, fast_rho, inv_stat, compact_stat, poly_rho)
    resident_supported = (T in (512, 1024, 2048) and D == 64 and io_is_bf16 and not poly_rho and
                          (kind == "softmax" or n == 16))
    if resident_bwd is True and not resident_supported:
        raise ValueError("resident backward needs bfloat16, T=512/1024/2048, D=64, "
                         "and softmax or exact asinh n=16")
    use_resident = (resident_supported and T == 2048 and bq == bk == 512 and compact_stat
                    if resident_bwd is None else bool(resident_bwd))
    if diagonal_bwd is True and not use_resident:
        raise ValueError("diagonal backward requires the resident backward backend")
    head_supported = (use_resident and T == 2048 and bq == bk == 512 and compact_stat)
    if head_resident is True and not head_supported:
        raise ValueError("whole-head residency needs resident bfloat16 T=2048,D=64, "
                         "512-square public tiles, and compact statistics")
    if range_guard and kind == "asinh" and n <= 32 and poly_rho:
        raise ValueError("range_guard is for exact radical evaluation")
    return var


def config_lists(kind, var: Variant, T: int, D: int, c: float, has_sink: bool, range_guard: bool):
    """The resolved variant and the wrapper constants (kernels/flash.py:823-856)
    as plain scalars: ints ``[kind, mode, n, fast_rho, inv_stat, has_sink]`` and
    floats ``[clamp, scale, guard_qk, guard_sink, guard_v]``."""
    unit = 1.0 if kind == "softmax" else float(c)
    guard_qk = guard_sink = guard_v = 0.0
    if kind == "asinh" and range_guard and var["n"] <= 32:
        bound = min(16.0, var["clamp"] / 2)
        mode = ALGX_MODE_GUARDED
        guard_qk = (bound / 1.01) ** 2
        guard_sink = bound / 1.01
        guard_v = min(1e8, 1e37 / ((T + int(has_sink)) * (2 * bound + 1) ** var["n"]))
    elif kind == "asinh":
        mode = ALGX_MODE_SHIFTED if var["shift"] else ALGX_MODE_CLIPPED
    else:
        mode = ALGX_MODE_SHIFTED
    ints = [ALGX_ATTN_SOFTMAX if kind == "softmax" else ALGX_ATTN_ASINH, mode, int(var["n"]),
            int(var["fast_rho"]), int(var["inv_stat"]), int(has_sink)]
    floats = [float(var["clamp"]), 1.0 / (math.sqrt(D) * unit), guard_qk, guard_sink, guard_v]
    return ints, floats


def sink_unit(kind: str, c: float) -> float:
    """The score unit the sink logit is divided by (kernels/flash.py:825-830)."""
    return 1.0 if kind == "softmax" else float(c)


def check_head_options(kind: str, n: int, h_shape, block_n: int):
    """The argument checks of ``fused_head`` (kernels/fused_head.py:269-272), in
    the reference's order, plus this build's tensor-core limits (alg_ce powers
    2..32, d a multiple of 64); ``h_shape`` is (N, d). Returns (N, d)."""
    if kind not in ("ce", "alg_ce"):
        raise ValueError(kind)
    if kind == "alg_ce" and (n & (n - 1)):
        raise ValueError("n must be a power of two")
    N, d = h_shape
    bn = min(block_n, N)
    if N % bn:
        raise ValueError(f"token count {N} must be divisible by block {bn}")
    if kind == "alg_ce" and n not in (2, 4, 8, 16, 32):
        raise ValueError("algx fused head supports alg_ce powers n in {2, 4, 8, 16, 32}")
    if d % 64:
        raise ValueError(f"algx fused head needs d to be a multiple of 64, got {d}")
    return N, d


def head_config_lists(kind: str, n: int, c: float, vocab: int, ignore_index=None):
    """The objective's constants as plain scalars: ints ``[kind, n, has_ignore,
    ignore_index]`` and floats ``[inv_c, clamp]`` (alg_ce clamp
    0.25 * (1e38 / V)^(1/n), kernels/fused_head.py:273)."""
    ints = [ALGX_HEAD_CE if kind == "ce" else ALGX_HEAD_ALG_CE, int(n), int(ignore_index is not None),
            int(ignore_index) if ignore_index is not None else 0]
    floats = [1.0 / float(c) if kind == "alg_ce" else 1.0,
              0.25 * _root(1e38 / vocab, n) if kind == "alg_ce" else 0.0]
    return ints, floats


def head_slope(kind: str, n: int, c: float) -> float:
    """d(objective)/d(logit) scale of the head backward (kernels/fused_head.py:247-254)."""
    return 1.0 if kind == "ce" else n / c


def check_qk_norm_options(shape, dim_last: int, gain_shape, x_is_supported: bool, gain_is_f32: bool, block: int,
                          eps: float):
    """The argument checks of ``qk_rms_norm`` (kernels/qk_norm.py:68-75)."""
    if len(shape) < 2 or dim_last != 64 or tuple(gain_shape) != (64,):
        raise ValueError("QK RMS kernel needs D=64 and a one-dimensional gain")
    if not x_is_supported or not gain_is_f32:
        raise ValueError("QK RMS kernel needs float32/BF16 input and float32 gain")
    rows = 1
    for s in shape[:-1]:
        rows *= int(s)
    if block < 8 or block % 8 or rows % block:
        raise ValueError("QK RMS row count must be divisible by a block aligned to eight rows")
    if eps <= 0:
        raise ValueError("QK RMS epsilon must be positive")
