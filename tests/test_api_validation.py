"""Argument validation mirrors the reference's ValueError conditions (CPU only)."""

import pytest
import torch

from algx.kernels.flash import flash_attention, make_variant
from algx.kernels.qk_norm import qk_rms_norm
from oracle import reference_math as R


def test_make_variant_matches_reference_rules():
    v = make_variant("asinh", 16, 8.0, 2048)
    assert not v["shift"] and v["inv_stat"] and v["fast_rho"]
    assert abs(v["clamp"] - R.attention_clamp(2048, 16)) < 1e-12
    with pytest.raises(ValueError, match="power of two"):
        make_variant("asinh", 12, 8.0, 2048)
    with pytest.raises(ValueError, match="positive and finite"):
        make_variant("asinh", 16, 0.0, 2048)
    with pytest.raises(ValueError, match="requires shift=False"):
        make_variant("asinh", 16, 8.0, 2048, shift=True, inv_stat=True)
    with pytest.raises(ValueError, match="unknown attention kernel"):
        make_variant("relu", 16, 8.0, 2048)
    with pytest.raises(ValueError, match="bounded radical"):
        make_variant("asinh", 8, 8.0, 2048, poly_rho=True)


def test_flash_rejects_like_reference():
    x = torch.ones((1, 1, 512, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="whole-head residency"):
        flash_attention(x, x, x, kind="asinh", c=8., head_resident=True)
    with pytest.raises(ValueError, match="divisible by blocks"):
        flash_attention(torch.ones((1, 1, 96, 64)), torch.ones((1, 1, 96, 64)), torch.ones((1, 1, 96, 64)),
                        kind="asinh", block=64)
    with pytest.raises(ValueError, match="resident backward"):
        f = torch.ones((1, 1, 256, 64))
        flash_attention(f, f, f, kind="asinh", resident_bwd=True)
    with pytest.raises(ValueError, match="diagonal backward"):
        f = torch.ones((1, 1, 256, 64))
        flash_attention(f, f, f, kind="asinh", diagonal_bwd=True)
    with pytest.raises(ValueError, match="head_dim 64"):
        f = torch.ones((1, 1, 256, 32))
        flash_attention(f, f, f, kind="asinh")


def test_flash_refuses_cpu_tensors():
    f = torch.ones((1, 1, 128, 64))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        flash_attention(f, f, f, kind="asinh", c=8.0)


def test_qk_norm_rejects_like_reference():
    g = torch.ones(64)
    with pytest.raises(ValueError, match="D=64"):
        qk_rms_norm(torch.ones((4, 32)), g)
    with pytest.raises(ValueError, match="float32 gain"):
        qk_rms_norm(torch.ones((1024, 64), dtype=torch.float16), g)
    with pytest.raises(ValueError, match="divisible by a block"):
        qk_rms_norm(torch.ones((100, 64)), g, block=8)
    with pytest.raises(ValueError, match="epsilon"):
        qk_rms_norm(torch.ones((1024, 64)), g, eps=0.0)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        qk_rms_norm(torch.ones((1024, 64)), g)
