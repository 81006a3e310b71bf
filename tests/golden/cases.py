"""Seeded input generators shared by the fixture generator and the tests.

Inputs are drawn with ``numpy.random.default_rng(seed)`` (PCG64), which is
reproducible across machines, so fixtures store only outputs plus an input
checksum that detects generator drift.
"""

import numpy as np
import torch


def normal(seed, shape, scale=1.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)


def uniform(seed, shape, lo=0.0, hi=1.0):
    rng = np.random.default_rng(seed)
    return rng.uniform(lo, hi, size=shape).astype(np.float32)


def integers(seed, shape, lo, hi):
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi, size=shape, dtype=np.int64)


def to_io(a, dtype):
    """float32 array -> float64 tensor holding values representable in ``dtype``."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype == torch.bfloat16:
        t = t.to(torch.bfloat16)
    return t.to(torch.float64)


# (name, n, c, with_sink, scale) attention fixture cases; shape (1, 2, 64, 64)
ATTN_SHAPE = (1, 2, 64, 64)
ATTN_CASES = [
    ("n16c8_sink", 16, 8.0, True, 1.0),
    ("n16c8_nosink", 16, 8.0, False, 1.0),
    ("n8c1_sink", 8, 1.0, True, 1.5),
    ("n32c8_nosink", 32, 8.0, False, 1.5),
]


def attn_inputs(seed, shape=ATTN_SHAPE, scale=1.0, with_sink=True):
    B, H, T, D = shape
    q = normal(seed, shape, scale)
    k = normal(seed + 1, shape, scale)
    v = normal(seed + 2, shape)
    g = normal(seed + 3, shape)
    sink = normal(seed + 4, (1, H, 1, 1), 0.5) if with_sink else None
    return q, k, v, g, sink


NORM_SHAPE = (2, 3, 16, 64)


def norm_inputs(seed, shape=NORM_SHAPE):
    x = normal(seed, shape, 3.0)
    x[0, 0, 0] = 0.0                      # an all-zero row, as in tests/test_qk_norm_tpu.py:21
    gain = (0.25 + 4.0 * uniform(seed + 1, (shape[-1],))).astype(np.float32)
    dy = normal(seed + 2, shape)
    return x, gain, dy


HEAD_SHAPE = (48, 64, 256)             # N tokens, d, V


def head_inputs(seed, shape=HEAD_SHAPE, e_scale=0.15):
    N, d, V = shape
    h = normal(seed, (N, d))
    e = normal(seed + 1, (V, d), e_scale)
    t = integers(seed + 2, (N,), 0, V)
    return h, e, t


# ---- optimizers (optimizers.py): a small parameter tree with every routing
# class (Muon matrices of three aspect ratios, the embedding, gains, sink) and
# three steps of gradients
# every routing class of optimizers.py:68-89: the embedding, gains, a sink, a
# bias, tall / square / wide matrices (two of one shape) and a 1-D "w_" vector
# (routed to Muon, which passes it through unorthogonalised)
OPTIM_SHAPES = {"bias": (8,), "embed": (10, 8), "ln1": (8,), "q_gain": (4,), "sink": (2,), "w_d": (16, 8),
                "w_k": (8, 8), "w_o": (8, 8), "w_q": (8, 16), "w_scale": (8,)}
OPTIM_DECAY = {"bias": False, "embed": True, "ln1": False, "q_gain": False, "sink": False, "w_d": True,
               "w_k": True, "w_o": True, "w_q": True, "w_scale": True}
OPTIM_ARGS = dict(lr=2e-2, weight_decay=0.1, total_steps=10, warmup_fraction=0.2, min_lr_ratio=0.1)
OPTIM_NS_SHAPES = [(8, 16), (16, 8), (12, 12), (3, 4, 6)]


def optim_inputs(seed):
    params = {k: normal(seed + i, s, 0.5) for i, (k, s) in enumerate(sorted(OPTIM_SHAPES.items()))}
    grads = [{k: normal(seed + 100 * (j + 1) + i, s, 0.1) for i, (k, s) in enumerate(sorted(OPTIM_SHAPES.items()))}
             for j in range(3)]
    return params, grads
