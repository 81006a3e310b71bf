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


def test_training_step_layers_validate_before_any_launch():
    """The training-step layers reject bad arguments, and CPU tensors, before any kernel call."""
    from algx._lib import AlgxError
    from algx.layers import add_rms_norm, aluglu, rms_norm, swiglu
    x = torch.ones((4, 768), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="float32 or bfloat16"):
        rms_norm(x.to(torch.float16), None)
    with pytest.raises(ValueError, match="gain must be float32"):
        rms_norm(x, torch.ones(767))
    with pytest.raises(ValueError, match="epsilon must be positive"):
        rms_norm(x, None, 0.0)
    with pytest.raises(ValueError, match="one shape and dtype"):
        add_rms_norm(x, torch.ones((4, 768)), None)
    with pytest.raises(ValueError, match="bfloat16"):
        swiglu(torch.ones((4, 64)))
    with pytest.raises(ValueError, match="multiple of 8"):
        aluglu(torch.ones((4, 24), dtype=torch.bfloat16))
    with pytest.raises(AlgxError, match="CUDA tensors only"):
        rms_norm(x, torch.ones(768))


def test_packed_attention_validates_its_layout():
    from algx.kernels.flash import qknorm_flash_attention_packed
    g = torch.ones(64)
    with pytest.raises(ValueError, match=r"\(B, T, 3, H, D\)"):
        qknorm_flash_attention_packed(torch.ones((1, 128, 2, 2, 64), dtype=torch.bfloat16), g, g)
    with pytest.raises(ValueError, match="head_dim 64"):
        qknorm_flash_attention_packed(torch.ones((1, 128, 3, 2, 32), dtype=torch.bfloat16), torch.ones(32),
                                      torch.ones(32))


def test_model_config_rejects_unsupported_choices():
    from algx.model import LMConfig
    with pytest.raises(ValueError, match="head_dim = 64"):
        LMConfig(d_model=768, n_heads=16).validate()
    with pytest.raises(ValueError, match="unknown ffn"):
        LMConfig(ffn="gelu").validate()
    with pytest.raises(ValueError, match="unknown position"):
        LMConfig(pos="none").validate()
    with pytest.raises(ValueError, match="unknown head"):
        LMConfig(head="mse").validate()
