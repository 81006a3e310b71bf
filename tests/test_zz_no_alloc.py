"""The allocation-free QK-norm backward agrees with the workspace version.

Some callers of this library cannot allocate device memory themselves: a
host framework that owns every device allocation and hands kernels only
fixed buffers, or code that runs while a caching pool allocator is locked.
For them, algx_qknorm_bwd_noalloc keeps its per-CTA dgain partials in a
static device array owned by the library instead of a caller workspace.

These tests call it through the C ABI twice in a row with different sizes
(so the second call cannot lean on what the first left in the shared
array) and compare dx and dgain with algx_qknorm_bwd, within the tolerances
the QK-norm parity tests use. The file is named to be collected last.
"""

import pytest
import torch

from algx import _lib as L

pytestmark = pytest.mark.gpu


def _inputs(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (3 * torch.randn(shape, device="cuda", generator=g)).to(dtype)
    dy = torch.randn(shape, device="cuda", generator=g).to(dtype)
    gain = 0.25 + 4 * torch.rand(64, device="cuda", generator=g)
    return x, dy, gain


def _with_workspace(x, dy, gain, eps):
    rows = x.numel() // 64
    dx, dg = torch.empty_like(x), torch.empty(64, device="cuda")
    nbytes = L.lib().algx_qknorm_bwd_workspace_size(rows, 64)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    L.check(L.lib().algx_qknorm_bwd(x.data_ptr(), gain.data_ptr(), dy.data_ptr(), dx.data_ptr(), dg.data_ptr(),
                                    rows, 64, L.dtype_code(x.dtype), eps, ws.data_ptr(), nbytes,
                                    torch.cuda.current_stream().cuda_stream), "algx_qknorm_bwd")
    return dx, dg


def _without_allocation(x, dy, gain, eps):
    rows = x.numel() // 64
    dx, dg = torch.empty_like(x), torch.empty(64, device="cuda")
    L.check(L.lib().algx_qknorm_bwd_noalloc(x.data_ptr(), gain.data_ptr(), dy.data_ptr(), dx.data_ptr(),
                                            dg.data_ptr(), rows, 64, L.dtype_code(x.dtype), eps,
                                            torch.cuda.current_stream().cuda_stream), "algx_qknorm_bwd_noalloc")
    return dx, dg


def _rel(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b).clamp_min(1e-30))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_noalloc_matches_workspace_entry_point_twice(dtype):
    eps = 1e-5
    # The first call spans the scratch array's full 256 CTAs; the second
    # needs fewer, so stale partial rows of the first call must not be read.
    for seed, shape in ((1, (4, 6, 2048, 64)), (2, (3, 5, 136, 64))):
        x, dy, gain = _inputs(shape, dtype, seed)
        dx_ref, dg_ref = _with_workspace(x, dy, gain, eps)
        dx, dg = _without_allocation(x, dy, gain, eps)
        torch.cuda.synchronize()
        # dx is computed row by row exactly as in the workspace version;
        # dgain differs only in the order of its fp32 partial sums.
        assert torch.equal(dx, dx_ref)
        assert _rel(dg, dg_ref) < 2e-6


def test_noalloc_rejects_rows_beyond_its_limit():
    x, dy, gain = _inputs((1, 1, 128, 64), torch.bfloat16, 3)
    dx, dg = torch.empty_like(x), torch.empty(64, device="cuda")
    status = L.lib().algx_qknorm_bwd_noalloc(x.data_ptr(), gain.data_ptr(), dy.data_ptr(), dx.data_ptr(),
                                             dg.data_ptr(), 2 ** 31, 64, L.ALGX_BF16, 1e-5,
                                             torch.cuda.current_stream().cuda_stream)
    assert status == L.ALGX_ERR_INVALID
    assert b"2147483647 rows" in L.lib().algx_last_error()
