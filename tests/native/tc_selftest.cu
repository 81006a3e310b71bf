// TEST-ONLY. One-CTA tcgen05 + TMA self-test of the operand layouts the
// attention and head kernels use; the host compares the result with a
// reference GEMM. Built into tests/native/libalgx_selftest.so (with the
// library's error and tensor-map helpers linked in privately), never into the
// product libalgx.so, and not part of the C ABI in include/algx.h:
//   int algx_selftest_tcgen05(int32_t mode, const void* a, const void* b,
//                             float* out, void* stream);
// a, b: bf16 device buffers, a (128 x ka, row-major; for mode 3 its
// transpose), b (nb x kb); out: fp32 128 x nout. The kernel's bounded waits
// report through this library's own algx_device_error().
//   mode 0: D[128x128]  = A[128x64]  . B[128x64]^T   (A, B K-major, SW128)
//   mode 1: D[128x64]   = A[128x128] . B[128x64]     (A K-major in two 64-wide
//                                                     chunks, B MN-major)
//   mode 2: same as 1 with A read from TMEM (bf16 pairs packed per column)
//   mode 3: same as 1 with A given transposed (MN-major A, two 64-row halves)
//   mode 4: D[128x256]  = A[128x64]  . B[256x64]^T   (N = 256)
#include "algx_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace algx {
namespace {

using namespace sm100;

constexpr int kSmemBytes = 200 * 1024;  // generous: a mis-strided operand stays inside the CTA

__global__ void __launch_bounds__(128) tc_selftest_kernel(const __grid_constant__ CUtensorMap ta,
                                                          const __grid_constant__ CUtensorMap tb, int mode,
                                                          const __nv_bfloat16* __restrict__ a_glob,
                                                          float* __restrict__ out, int* dev_err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + 32768;
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bar_load, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb_ = tmem_base;
  const int ncols = mode == 0 ? 128 : (mode == 4 ? 256 : 64);

  if (threadIdx.x == 0) {
    if (mode == 0) {
      mbar_expect_tx(&bar_load, 2 * 16384);
      tma_load_2d(sa, &ta, &bar_load, 0, 0);
      tma_load_2d(sb, &tb, &bar_load, 0, 0);
    } else if (mode == 1 || mode == 3) {
      mbar_expect_tx(&bar_load, 3 * 16384);
      tma_load_2d(sa, &ta, &bar_load, 0, 0);
      tma_load_2d(sa + 16384, &ta, &bar_load, 64, 0);
      tma_load_2d(sb, &tb, &bar_load, 0, 0);
    } else if (mode == 2) {
      mbar_expect_tx(&bar_load, 16384);
      tma_load_2d(sb, &tb, &bar_load, 0, 0);
    } else {
      mbar_expect_tx(&bar_load, 16384 + 32768);
      tma_load_2d(sa, &ta, &bar_load, 0, 0);
      tma_load_2d(sb, &tb, &bar_load, 0, 0);
    }
  }
  if (mode == 2) {
    // Row r of A (128 bf16) -> TMEM lane r, columns 256 + [0, 64): pairs packed low = even k.
    const int r = threadIdx.x;
    for (int c0 = 0; c0 < 64; c0 += 16) {
      uint32_t vals[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int kk = 2 * (c0 + i);
        vals[i] = pack_bf16x2(__bfloat162float(a_glob[r * 128 + kk]), __bfloat162float(a_glob[r * 128 + kk + 1]));
      }
      tmem_st16(tb_ + ((uint32_t)(warp * 32) << 16) + 256 + c0, vals);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  bool ok = mbar_wait_warp(&bar_load, 0, &abort_flag, dev_err);
  if (threadIdx.x == 0 && ok) {
    tc_fence_after();
    const uint32_t a0 = smem_u32(sa), b0 = smem_u32(sb);
    if (mode == 0 || mode == 4) {
      const uint32_t id = idesc_bf16_f32(128, ncols, 0, 0);
      for (int k = 0; k < 4; ++k)
        mma_ss(tb_, desc_sw128(a0 + k * 32, 16, 1024), desc_sw128(b0 + k * 32, 16, 1024), id, k > 0);
    } else if (mode == 1) {
      const uint32_t id = idesc_bf16_f32(128, 64, 0, 1);
      for (int k = 0; k < 8; ++k)
        mma_ss(tb_, desc_sw128(a0 + (k / 4) * 16384 + (k % 4) * 32, 16, 1024), desc_sw128(b0 + k * 2048, 8192, 1024),
               id, k > 0);
    } else if (mode == 2) {
      const uint32_t id = idesc_bf16_f32(128, 64, 0, 1);
      for (int k = 0; k < 8; ++k) mma_ts(tb_, tb_ + 256 + k * 8, desc_sw128(b0 + k * 2048, 8192, 1024), id, k > 0);
    } else {
      const uint32_t id = idesc_bf16_f32(128, 64, 1, 1);
      for (int k = 0; k < 8; ++k)
        mma_ss(tb_, desc_sw128(a0 + k * 2048, 16384, 1024), desc_sw128(b0 + k * 2048, 8192, 1024), id, k > 0);
    }
    mma_commit(&bar_mma);
  }
  __syncthreads();
  ok = mbar_wait_warp(&bar_mma, 0, &abort_flag, dev_err) && ok;
  tc_fence_after();
  if (ok) {
    const int row = threadIdx.x;
    for (int c0 = 0; c0 < ncols; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tb_ + ((uint32_t)(warp * 32) << 16) + c0, r);
#pragma unroll
      for (int i = 0; i < 32; ++i) out[row * ncols + c0 + i] = __uint_as_float(r[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb_, 512);
}

}  // namespace
}  // namespace algx

using namespace algx;

extern "C" __attribute__((visibility("default"))) int algx_selftest_tcgen05(int32_t mode, const void* a, const void* b, float* out, void* stream) {
  ALGX_REQUIRE(mode >= 0 && mode <= 4, "selftest: mode must be 0..4");
  ALGX_REQUIRE(a && b && out, "selftest: NULL pointer");
  CUtensorMap ta, tb;
  const bool wide_a = mode == 1 || mode == 2 || mode == 3;
  if (int s = make_tmap_2d(&ta, a, ALGX_BF16, wide_a ? 128 : 64, 128, wide_a ? 256 : 128, 64, 128, true)) return s;
  const uint32_t brows = mode == 4 ? 256 : 128;
  if (int s = make_tmap_2d(&tb, b, ALGX_BF16, 64, brows, 128, 64, brows, true)) return s;
  ALGX_CUDA(cudaFuncSetAttribute(tc_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  int* err = device_error_word();
  tc_selftest_kernel<<<1, 128, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
      ta, tb, mode, static_cast<const __nv_bfloat16*>(a), out, err);
  ALGX_LAUNCHED("selftest launch");
  return ALGX_OK;
}
