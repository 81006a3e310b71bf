// QK RMS norm forward and backward, D = 64 (kernels/qk_norm.py:62-76 and
// algebraic.py:76-83). HBM-bound: 128-bit loads/stores, TPR threads per row
// (8 for bf16, 16 for fp32), row reductions by warp shuffles, a fixed grid
// of a few CTAs per SM looping over rows. dgain is reduced deterministically:
// per-CTA column partials in a workspace, then one fixed-order sum.
#include <mutex>

#include "algx_common.cuh"
#include "vec_io.cuh"

namespace algx {
namespace {

constexpr int kDim = 64;
constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kMaxBlocks = 148 * 4;

template <typename T>
__global__ void __launch_bounds__(kThreads) qknorm_fwd_kernel(const T* __restrict__ x,
                                                              const float* __restrict__ gain,
                                                              T* __restrict__ y, int64_t rows, float eps) {
  using V = Vec<T>;
  const int lane = threadIdx.x & 31;
  const int sub = lane % V::TPR;
  const int rl = lane / V::TPR;
  float g[V::N];
#pragma unroll
  for (int i = 0; i < V::N; ++i) g[i] = gain[sub * V::N + i];
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  for (int64_t r0 = w * V::RPW * kUnroll; r0 < rows; r0 += warps * V::RPW * kUnroll) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      raw[u] = row < rows ? ld_stream(x + row * kDim + sub * V::N) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      float v[V::N];
      unpack<T>(raw[u], v);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) ss = fmaf(v[i], v[i], ss);
      ss = row_sum<V::TPR>(ss);
      const float tau = rsqrtf(ss * (1.0f / kDim) + eps);
#pragma unroll
      for (int i = 0; i < V::N; ++i) v[i] = (v[i] * tau) * g[i];
      if (row < rows) *reinterpret_cast<uint4*>(y + row * kDim + sub * V::N) = pack<T>(v);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) qknorm_bwd_kernel(const T* __restrict__ x,
                                                              const float* __restrict__ gain,
                                                              const T* __restrict__ dy, T* __restrict__ dx,
                                                              float* __restrict__ partial, int64_t rows,
                                                              float eps) {
  using V = Vec<T>;
  __shared__ float red[kThreads][V::N + 1];
  const int lane = threadIdx.x & 31;
  const int sub = lane % V::TPR;
  const int rl = lane / V::TPR;
  float g[V::N], acc[V::N];
#pragma unroll
  for (int i = 0; i < V::N; ++i) {
    g[i] = gain[sub * V::N + i];
    acc[i] = 0.f;
  }
  const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  for (int64_t r0 = w * V::RPW * kUnroll; r0 < rows; r0 += warps * V::RPW * kUnroll) {
    uint4 rx[kUnroll], rd[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      const bool ok = row < rows;
      rx[u] = ok ? ld_stream(x + row * kDim + sub * V::N) : make_uint4(0, 0, 0, 0);
      rd[u] = ok ? ld_stream(dy + row * kDim + sub * V::N) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      float xv[V::N], dv[V::N];
      unpack<T>(rx[u], xv);
      unpack<T>(rd[u], dv);
      float ss = 0.f, sdg = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) {
        ss = fmaf(xv[i], xv[i], ss);
        sdg = fmaf(dv[i] * g[i], xv[i], sdg);
      }
      ss = row_sum<V::TPR>(ss);
      sdg = row_sum<V::TPR>(sdg);
      const float tau = rsqrtf(ss * (1.0f / kDim) + eps);
      const float corr = tau * tau * tau * sdg * (1.0f / kDim);
      float out[V::N];
#pragma unroll
      for (int i = 0; i < V::N; ++i) {
        out[i] = (dv[i] * g[i]) * tau - xv[i] * corr;
        acc[i] = fmaf(dv[i], xv[i] * tau, acc[i]);
      }
      if (row < rows) *reinterpret_cast<uint4*>(dx + row * kDim + sub * V::N) = pack<T>(out);
    }
  }
#pragma unroll
  for (int i = 0; i < V::N; ++i) red[threadIdx.x][i] = acc[i];
  __syncthreads();
  if (threadIdx.x < kDim) {
    const int c = threadIdx.x, s = c / V::N, i = c % V::N;
    float sum = 0.f;
    for (int t = s; t < kThreads; t += V::TPR) sum += red[t][i];
    partial[(int64_t)blockIdx.x * kDim + c] = sum;
  }
}

// dgain[c] = sum_b partial[b][c]: 16 strided partial sums per column, then a
// fixed-order sum of the 16 (deterministic for a given grid size).
constexpr int kReduceThreads = 1024;
__global__ void __launch_bounds__(kReduceThreads) qknorm_dgain_reduce(const float* __restrict__ partial, int nblocks,
                                                                      float* __restrict__ dgain) {
  __shared__ float red[kReduceThreads / kDim][kDim];
  const int c = threadIdx.x % kDim, p = threadIdx.x / kDim;
  float s = 0.f;
  for (int b = p; b < nblocks; b += kReduceThreads / kDim) s += partial[(int64_t)b * kDim + c];
  red[p][c] = s;
  __syncthreads();
  if (threadIdx.x < kDim) {
    float t = 0.f;
    for (int i = 0; i < kReduceThreads / kDim; ++i) t += red[i][threadIdx.x];
    dgain[threadIdx.x] = t;
  }
}

template <typename T>
int grid_for(int64_t rows) {
  const int64_t per_block = (int64_t)(kThreads / 32) * Vec<T>::RPW * kUnroll;
  int64_t g = (rows + per_block - 1) / per_block;
  if (g > kMaxBlocks) g = kMaxBlocks;
  return (int)(g < 1 ? 1 : g);
}

// Scratch of algx_qknorm_bwd_noalloc: one row of kDim fp32 dgain partials per
// CTA, for at most kNoAllocBlocks CTAs (64 KiB per device, held by every GPU
// that loads the library until the process exits). Host code must not pass
// the symbol itself to a kernel: its device address comes from
// cudaGetSymbolAddress, taken once per device in noalloc_scratch().
constexpr int kNoAllocBlocks = 256;
constexpr int64_t kNoAllocMaxRows = 2147483647;  // rows beyond int32 range are rejected
static __device__ __align__(256) float g_noalloc_partials[kNoAllocBlocks * kDim];

int noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = 0;
  ALGX_CUDA(cudaGetDevice(&dev));
  ALGX_REQUIRE(dev >= 0 && dev < 64, "qknorm_bwd_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    ALGX_CUDA(cudaGetSymbolAddress(&p, g_noalloc_partials));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return ALGX_OK;
}

int check_args(const void* x, const float* gain, const void* y, int64_t rows, int64_t dim, int32_t dtype,
               float eps) {
  ALGX_REQUIRE(x && gain && y, "qknorm: NULL pointer");
  ALGX_REQUIRE(dim == kDim, "QK RMS kernel needs D=64 and a one-dimensional gain");
  ALGX_REQUIRE(dtype == ALGX_F32 || dtype == ALGX_BF16, "QK RMS kernel needs float32/BF16 input and float32 gain");
  ALGX_REQUIRE(rows >= 0, "qknorm: negative row count");
  ALGX_REQUIRE(eps > 0.f, "QK RMS epsilon must be positive");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0,
               "qknorm: tensors must be 16-byte aligned");
  return ALGX_OK;
}

}  // namespace
}  // namespace algx

using namespace algx;

extern "C" {

int algx_qknorm_fwd(const void* x, const float* gain, void* y, int64_t rows, int64_t dim, int32_t dtype,
                    float eps, void* stream) {
  if (int s = check_args(x, gain, y, rows, dim, dtype, eps)) return s;
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == ALGX_BF16) {
    qknorm_fwd_kernel<__nv_bfloat16><<<grid_for<__nv_bfloat16>(rows), kThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), gain, static_cast<__nv_bfloat16*>(y), rows, eps);
  } else {
    qknorm_fwd_kernel<float><<<grid_for<float>(rows), kThreads, 0, st>>>(
        static_cast<const float*>(x), gain, static_cast<float*>(y), rows, eps);
  }
  ALGX_LAUNCHED("qknorm_fwd launch");
  return ALGX_OK;
}

size_t algx_qknorm_bwd_workspace_size(int64_t rows, int64_t dim) {
  (void)dim;
  const int g = grid_for<float>(rows) > grid_for<__nv_bfloat16>(rows) ? grid_for<float>(rows)
                                                                      : grid_for<__nv_bfloat16>(rows);
  return (size_t)g * kDim * sizeof(float);
}

int algx_qknorm_bwd(const void* x, const float* gain, const void* dy, void* dx, float* dgain, int64_t rows,
                    int64_t dim, int32_t dtype, float eps, void* workspace, size_t workspace_bytes,
                    void* stream) {
  if (int s = check_args(x, gain, dx, rows, dim, dtype, eps)) return s;
  ALGX_REQUIRE(dy && dgain, "qknorm_bwd: NULL pointer");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(dy) & 15) == 0, "qknorm: tensors must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    ALGX_CUDA(cudaMemsetAsync(dgain, 0, kDim * sizeof(float), st));
    return ALGX_OK;
  }
  const int grid = dtype == ALGX_BF16 ? grid_for<__nv_bfloat16>(rows) : grid_for<float>(rows);
  ALGX_REQUIRE(workspace && workspace_bytes >= (size_t)grid * kDim * sizeof(float),
               "qknorm_bwd: workspace too small (see algx_qknorm_bwd_workspace_size)");
  float* partial = static_cast<float*>(workspace);
  if (dtype == ALGX_BF16) {
    qknorm_bwd_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), gain, static_cast<const __nv_bfloat16*>(dy),
        static_cast<__nv_bfloat16*>(dx), partial, rows, eps);
  } else {
    qknorm_bwd_kernel<float><<<grid, kThreads, 0, st>>>(static_cast<const float*>(x), gain,
                                                        static_cast<const float*>(dy), static_cast<float*>(dx),
                                                        partial, rows, eps);
  }
  ALGX_LAUNCHED("qknorm_bwd launch");
  qknorm_dgain_reduce<<<1, kReduceThreads, 0, st>>>(partial, grid, dgain);
  ALGX_LAUNCHED("qknorm_dgain_reduce launch");
  return ALGX_OK;
}

// The same backward as algx_qknorm_bwd, for callers that cannot allocate
// device memory: its dgain partials live in g_noalloc_partials instead of a
// caller workspace. See include/algx.h for the contract.
int algx_qknorm_bwd_noalloc(const void* x, const float* gain, const void* dy, void* dx, float* dgain, int64_t rows,
                            int64_t dim, int32_t dtype, float eps, void* stream) {
  if (int s = check_args(x, gain, dx, rows, dim, dtype, eps)) return s;
  ALGX_REQUIRE(dy && dgain, "qknorm_bwd_noalloc: NULL pointer");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(dy) & 15) == 0, "qknorm: tensors must be 16-byte aligned");
  ALGX_REQUIRE(rows <= kNoAllocMaxRows,
               "qknorm_bwd_noalloc: at most 2147483647 rows (use algx_qknorm_bwd with a workspace)");
  float* partial = nullptr;
  if (int s = noalloc_scratch(&partial)) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    ALGX_CUDA(cudaMemsetAsync(dgain, 0, kDim * sizeof(float), st));
    return ALGX_OK;
  }
  // Every CTA of the grid writes its whole partial row, so nothing in the
  // scratch needs clearing; the reduction reads exactly those rows.
  int grid = dtype == ALGX_BF16 ? grid_for<__nv_bfloat16>(rows) : grid_for<float>(rows);
  if (grid > kNoAllocBlocks) grid = kNoAllocBlocks;
  if (dtype == ALGX_BF16) {
    qknorm_bwd_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), gain, static_cast<const __nv_bfloat16*>(dy),
        static_cast<__nv_bfloat16*>(dx), partial, rows, eps);
  } else {
    qknorm_bwd_kernel<float><<<grid, kThreads, 0, st>>>(static_cast<const float*>(x), gain,
                                                        static_cast<const float*>(dy), static_cast<float*>(dx),
                                                        partial, rows, eps);
  }
  ALGX_LAUNCHED("qknorm_bwd_noalloc launch");
  qknorm_dgain_reduce<<<1, kReduceThreads, 0, st>>>(partial, grid, dgain);
  ALGX_LAUNCHED("qknorm_dgain_reduce launch");
  return ALGX_OK;
}

}  // extern "C"
