"""tcgen05 / TMA operand-layout self-test on the B200 (one CTA per mode).

The kernel lives in the test-only library tests/native/libalgx_selftest.so,
built by the same Makefile as libalgx.so but not part of it.
"""

import ctypes
import os

import pytest
import torch

from tests.gpu_util import dump

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "native", "libalgx_selftest.so")


def _selftest_lib():
    if not os.path.exists(LIB):
        raise FileNotFoundError(f"{LIB} is missing: build it with __graft_entry__.build()")
    h = ctypes.CDLL(LIB)
    h.algx_selftest_tcgen05.argtypes = [ctypes.c_int32] + [ctypes.c_void_p] * 4
    h.algx_selftest_tcgen05.restype = ctypes.c_int
    h.algx_device_error.argtypes = [ctypes.POINTER(ctypes.c_int32)]
    h.algx_device_error.restype = ctypes.c_int
    h.algx_last_error.restype = ctypes.c_char_p
    return h


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_tcgen05_layouts(mode):
    lib = _selftest_lib()
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
    status = lib.algx_selftest_tcgen05(mode, a.data_ptr(), b.data_ptr(), out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    assert status == 0, lib.algx_last_error()
    torch.cuda.synchronize()
    err = ctypes.c_int32(0)
    assert lib.algx_device_error(ctypes.byref(err)) == 0 and err.value == 0
    if not torch.allclose(out, ref, atol=1e-2, rtol=1e-3):
        dump(f"selftest_mode{mode}", a=a, b=b, out=out, ref=ref)
    torch.testing.assert_close(out, ref, atol=1e-2, rtol=1e-3)
