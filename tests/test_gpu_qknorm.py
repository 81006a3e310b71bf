"""QK-norm kernels vs the oracle (cases of tests/test_qk_norm_tpu.py:21-43)."""

import pytest
import torch

from algx.kernels.qk_norm import qk_rms_norm
from oracle import reference_math as R
from tests.gpu_util import rel_l2

pytestmark = pytest.mark.gpu


def _inputs(dtype, shape=(2, 3, 512, 64), seed=181):
    g = torch.Generator().manual_seed(seed)
    x = 3 * torch.randn(shape, generator=g)
    x[0, 0, 0] = 0.0
    gain = 0.25 + 4 * torch.rand(64, generator=g)
    do = torch.randn(shape, generator=g)
    return x.to(dtype), gain, do.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("block", [256, 1024])
@pytest.mark.parametrize("eps", [1e-5, 1e-3])
def test_qk_norm_output_and_vjp(dtype, block, eps):
    x, gain, do = _inputs(dtype)
    xc = x.cuda().requires_grad_(True)
    gc = gain.cuda().requires_grad_(True)
    y = qk_rms_norm(xc, gc, eps, block=block)
    torch.sum(y.float() * do.cuda().float()).backward()
    io = None if dtype == torch.float32 else torch.bfloat16
    y_ref = R.rms_norm(x.double(), gain.double(), eps, io_dtype=io)
    dx_ref, dg_ref = R.qk_norm_backward(x.double(), gain.double(), do.double(), eps)
    tol = 2e-6 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(y.detach().double().cpu(), y_ref, atol=tol, rtol=tol)
    # dx leaves the kernel in the I/O dtype: compare with the oracle rounded the same way.
    dx_cmp = dx_ref if io is None else dx_ref.to(io).double()
    gtol = 2e-6 if dtype == torch.float32 else 1e-3
    assert torch.isfinite(xc.grad.float()).all()
    assert rel_l2(xc.grad, dx_cmp) < gtol
    assert rel_l2(gc.grad, dg_ref) < gtol


def test_qk_norm_large_rows_and_ragged_tail():
    """Row counts that are not a multiple of the kernel's per-block rows."""
    x, gain, do = _inputs(torch.bfloat16, shape=(3, 5, 1000 + 8, 64), seed=5)
    xc = x.cuda().requires_grad_(True)
    gc = gain.cuda().requires_grad_(True)
    y = qk_rms_norm(xc, gc, 1e-5, block=8)
    torch.sum(y.float() * do.cuda().float()).backward()
    y_ref = R.rms_norm(x.double(), gain.double(), 1e-5, io_dtype=torch.bfloat16)
    assert rel_l2(y.detach(), y_ref) < 4e-3
    _, dg_ref = R.qk_norm_backward(x.double(), gain.double(), do.double(), 1e-5)
    assert rel_l2(gc.grad, dg_ref) < 1e-4
