"""tcgen05 / TMA operand-layout self-test on the B200 (one CTA per mode)."""

import pytest
import torch

from algx import _lib as L
from tests.gpu_util import dump

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_tcgen05_layouts(mode):
    torch.manual_seed(100 + mode)
    dev = "cuda"
    bf = torch.bfloat16
    if mode == 0:
        a, b = torch.randn(128, 64, device=dev).to(bf), torch.randn(128, 64, device=dev).to(bf)
        ref = a.float() @ b.float().T
    elif mode in (1, 2):
        a, b = torch.randn(128, 128, device=dev).to(bf), torch.randn(128, 64, device=dev).to(bf)
        ref = a.float() @ b.float()
    elif mode == 3:
        a, b = torch.randn(128, 128, device=dev).to(bf), torch.randn(128, 64, device=dev).to(bf)
        ref = a.float().T @ b.float()
    else:
        a, b = torch.randn(128, 64, device=dev).to(bf), torch.randn(256, 64, device=dev).to(bf)
        ref = a.float() @ b.float().T
    out = torch.full_like(ref, float("nan"))
    L.check(L.lib().algx_selftest_tcgen05(mode, a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream), "selftest")
    torch.cuda.synchronize()
    assert L.device_error() == 0
    if not torch.allclose(out, ref, atol=1e-2, rtol=1e-3):
        dump(f"selftest_mode{mode}", a=a, b=b, out=out, ref=ref)
    torch.testing.assert_close(out, ref, atol=1e-2, rtol=1e-3)
