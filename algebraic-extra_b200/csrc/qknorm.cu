// QK RMS norm forward and backward, D = 64 (kernels/qk_norm.py:62-76 and
// algebraic.py:76-83). HBM-bound: 128-bit loads/stores, TPR threads per row
// (8 for bf16, 16 for fp32), row reductions by warp shuffles, a fixed grid
// of a few CTAs per SM looping over rows. dgain is reduced deterministically:
// per-CTA column partials in a workspace, then one fixed-order sum.
#include <algorithm>
#include <mutex>

#include "algx_common.cuh"
#include "sm100.cuh"
#include "tmap.h"
#include "vec_io.cuh"

namespace algx {
namespace {

constexpr int kDim = 64;
constexpr int kThreads = 256;
constexpr int kUnroll = 4;   // rows per thread in flight, forward
constexpr int kUnrollB = 2;  // backward (two loads per row; 4 CTAs per SM within 64 registers)
constexpr int kMaxBlocks = 148 * 4;

template <typename T>
__global__ void __launch_bounds__(kThreads, kMaxBlocks / 148) qknorm_fwd_kernel(const T* __restrict__ x,
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

// Four CTAs per SM (kMaxBlocks = 4 x 148) must be resident at once: the
// register bound keeps the grid in one wave.
template <typename T>
__global__ void __launch_bounds__(kThreads, kMaxBlocks / 148) qknorm_bwd_kernel(const T* __restrict__ x,
                                                              const float* __restrict__ gain,
                                                              const T* __restrict__ dy, T* __restrict__ dx,
                                                              float* __restrict__ partial, int64_t rows,
                                                              float eps) {
  using V = Vec<T>;
  __shared__ float red[kThreads][V::N + 1];
  pdl_trigger();  // the dgain reduction may be scheduled now; it waits for this grid to finish
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
  for (int64_t r0 = w * V::RPW * kUnrollB; r0 < rows; r0 += warps * V::RPW * kUnrollB) {
    uint4 rx[kUnrollB], rd[kUnrollB];
#pragma unroll
    for (int u = 0; u < kUnrollB; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      const bool ok = row < rows;
      rx[u] = ok ? ld_stream(x + row * kDim + sub * V::N) : make_uint4(0, 0, 0, 0);
      rd[u] = ok ? ld_stream(dy + row * kDim + sub * V::N) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnrollB; ++u) {
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
    partial[(int64_t)c * gridDim.x + blockIdx.x] = sum;  // column-major: one contiguous row per column
  }
}

// Backward with the rows staged through shared memory: one CTA per SM, a
// producer thread streams 16 KB chunks of x and dy with bulk asynchronous
// copies into a kStagesB-deep ring (so up to 192 KB per SM are in flight
// whatever the consumers are doing), and 16 consumer warps apply the per-row
// maths of qknorm_bwd_kernel (dx bit-identical) and write dx with 16-byte
// stores. Chunk c of the rows goes to CTA c % gridDim.x. dgain partials as
// in qknorm_bwd_kernel (column-major, one per CTA and column).
constexpr int kChunkBytesB = 16384;
constexpr int kStagesB = 6;
constexpr int kConsumerWarpsB = 16;
constexpr int kThreadsB = (kConsumerWarpsB + 1) * 32;
constexpr int kSmemB = 2 * kStagesB * kChunkBytesB;
constexpr int kMaxBlocksB = 256;  // grid cap (one CTA per SM up to this many SMs); sizes the workspace

template <typename T>
__global__ void __launch_bounds__(kThreadsB, 1)
    qknorm_bwd_staged_kernel(const T* __restrict__ x, const float* __restrict__ gain, const T* __restrict__ dy,
                             T* __restrict__ dx, float* __restrict__ partial, int64_t rows, float eps, int* dev_err) {
  using V = Vec<T>;
  using namespace sm100;
  constexpr int kRowsPerChunk = kChunkBytesB / (kDim * (int)sizeof(T));
  extern __shared__ __align__(128) uint8_t smem_b[];
  __shared__ uint64_t full[kStagesB], empty[kStagesB];
  __shared__ float red[kConsumerWarpsB * 32][V::N + 1];
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  pdl_trigger();  // the dgain reduction may be scheduled now; it waits for this grid to finish
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nchunks = (rows + kRowsPerChunk - 1) / kRowsPerChunk;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStagesB; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarpsB);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  __syncthreads();
  // launched as a programmatic dependent: the set-up above overlapped the
  // previous kernel's tail; its results (x, dy, gain, the workspace) are
  // read only after it has finished
  pdl_wait();
  if (warp == kConsumerWarpsB) {
    // ----- producer: chunk bytes of x and dy per stage
    if (lane == 0) {
      int it = 0;
      int pending[kStagesB];
      for (int i = 0; i < kStagesB; ++i) pending[i] = -1;
      for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x, ++it) {
        const int s = it % kStagesB;
        if (it >= kStagesB && !mbar_wait(&empty[s], ((it / kStagesB) - 1) & 1, abort_v, dev_err)) break;
        const int64_t r0 = c * kRowsPerChunk;
        const int64_t nr = rows - r0 < kRowsPerChunk ? rows - r0 : kRowsPerChunk;
        const uint32_t bytes = (uint32_t)(nr * kDim * sizeof(T));
        uint8_t* st = smem_b + (size_t)s * 2 * kChunkBytesB;
        mbar_expect_tx(&full[s], 2 * bytes);
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(st)),
                     "l"(x + r0 * kDim), "r"(bytes), "r"(smem_u32(&full[s]))
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(st + kChunkBytesB)),
                     "l"(dy + r0 * kDim), "r"(bytes), "r"(smem_u32(&full[s]))
                     : "memory");
        pending[s] = it;
      }
      if (*abort_v) {  // let copies in flight land before the CTA exits
        volatile int quiet = 0;
        for (int i = 0; i < kStagesB; ++i)
          if (pending[i] >= 0) mbar_wait(&full[i], (pending[i] / kStagesB) & 1, &quiet, nullptr);
      }
    }
  } else {
    // ----- consumers: warp w takes rows w*RPW + rl (+ 16 RPW ...) of each chunk
    const int sub = lane % V::TPR, rl = lane / V::TPR;
    float g[V::N], acc[V::N];
#pragma unroll
    for (int i = 0; i < V::N; ++i) {
      g[i] = gain[sub * V::N + i];
      acc[i] = 0.f;
    }
    int it = 0;
    for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x, ++it) {
      const int s = it % kStagesB;
      if (!mbar_wait_warp(&full[s], (it / kStagesB) & 1, abort_v, dev_err)) break;
      const uint8_t* st = smem_b + (size_t)s * 2 * kChunkBytesB;
      const int64_t r0 = c * kRowsPerChunk;
#pragma unroll
      for (int p = 0; p < kRowsPerChunk / (kConsumerWarpsB * V::RPW); ++p) {
        const int lr = (p * kConsumerWarpsB + warp) * V::RPW + rl;  // row within the chunk
        const int64_t row = r0 + lr;
        const bool ok = row < rows;
        const uint4 rx = ok ? *reinterpret_cast<const uint4*>(st + (size_t)lr * kDim * sizeof(T) + sub * 16)
                            : make_uint4(0, 0, 0, 0);
        const uint4 rd = ok ? *reinterpret_cast<const uint4*>(st + kChunkBytesB + (size_t)lr * kDim * sizeof(T) +
                                                              sub * 16)
                            : make_uint4(0, 0, 0, 0);
        float xv[V::N], dv[V::N];
        unpack<T>(rx, xv);
        unpack<T>(rd, dv);
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
        if (ok) *reinterpret_cast<uint4*>(dx + row * kDim + sub * V::N) = pack<T>(out);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int i = 0; i < V::N; ++i) red[threadIdx.x][i] = acc[i];
  }
  __syncthreads();
  if (threadIdx.x < kDim) {
    const int c = threadIdx.x, sb = c / V::N, i = c % V::N;
    float sum = 0.f;
    for (int t = sb; t < kConsumerWarpsB * 32; t += V::TPR) sum += red[t][i];
    partial[(int64_t)c * gridDim.x + blockIdx.x] = sum;
  }
}

// dgain[c] = sum_b partial[c][b]: one warp per column, lane l summing blocks
// l, l + 32, ... in order, then a fixed butterfly over the lanes
// (deterministic for a given grid size); 64 warps in two CTAs. A lane's (at
// most eight) loads are issued together before the in-order sum. It lets the
// next kernel of the stream launch at once (a row kernel launched as its
// programmatic dependent waits in pdl_wait() until this grid has finished).
constexpr int kReduceThreads = 1024;
__global__ void __launch_bounds__(kReduceThreads) qknorm_dgain_reduce(const float* __restrict__ partial, int nblocks,
                                                                      float* __restrict__ dgain) {
  pdl_trigger();  // the next kernel may be scheduled now; it waits for this grid to finish
  pdl_wait();     // launched as a programmatic dependent of the row kernel: its partials are complete
  const int c = blockIdx.x * (kReduceThreads / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (c >= kDim) return;
  const float* col = partial + (int64_t)c * nblocks;
  float s = 0.f;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = lane + 32 * j < nblocks ? col[lane + 32 * j] : 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) s += v[j];
  for (int b = lane + 256; b < nblocks; b += 32) s += col[b];  // grids above 256 CTAs (none launched today)
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) dgain[c] = s;
}
constexpr int kReduceBlocks = kDim / (kReduceThreads / 32);

template <typename T>
int grid_for(int64_t rows) {
  const int64_t per_block = (int64_t)(kThreads / 32) * Vec<T>::RPW * kUnroll;
  int64_t g = (rows + per_block - 1) / per_block;
  if (g > kMaxBlocks) g = kMaxBlocks;
  return (int)(g < 1 ? 1 : g);
}

// Scratch of algx_qknorm_bwd_noalloc: kDim fp32 dgain partials per CTA (column
// by column), for at most kNoAllocBlocks CTAs (64 KiB per device, held by every GPU
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
  // the staged kernel's grid: one CTA per chunk (fp32 chunks hold the fewest rows), at most kMaxBlocksB
  const int64_t chunk_rows = kChunkBytesB / (kDim * (int64_t)sizeof(float));
  const int64_t g = std::max<int64_t>(1, std::min<int64_t>((rows + chunk_rows - 1) / chunk_rows, kMaxBlocksB));
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
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(dx) & 15) == 0, "qknorm: tensors must be 16-byte aligned");
  int dev = 0, sms = 0;
  ALGX_CUDA(cudaGetDevice(&dev));
  ALGX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t chunk_rows = kChunkBytesB / (kDim * (dtype == ALGX_BF16 ? 2 : 4));
  const int grid = (int)std::min<int64_t>(std::min<int64_t>((rows + chunk_rows - 1) / chunk_rows, sms),
                                          kMaxBlocksB);  // one CTA per SM
  ALGX_REQUIRE(workspace && workspace_bytes >= (size_t)grid * kDim * sizeof(float),
               "qknorm_bwd: workspace too small (see algx_qknorm_bwd_workspace_size)");
  float* partial = static_cast<float*>(workspace);
  auto run = [&](auto kern, auto tag) -> int {
    using TT = decltype(tag);
    ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemB));
    ALGX_CUDA(launch_dependent(kern, grid, kThreadsB, kSmemB, st, static_cast<const TT*>(x), gain,
                               static_cast<const TT*>(dy), static_cast<TT*>(dx), partial, rows, eps,
                               device_error_word()));
    ALGX_LAUNCHED("qknorm_bwd launch");
    return ALGX_OK;
  };
  if (int s = dtype == ALGX_BF16 ? run(qknorm_bwd_staged_kernel<__nv_bfloat16>, __nv_bfloat16{})
                                 : run(qknorm_bwd_staged_kernel<float>, float{}))
    return s;
  ALGX_CUDA(launch_dependent(qknorm_dgain_reduce, kReduceBlocks, kReduceThreads, 0, st, partial, grid, dgain));
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
  // Every CTA of the grid writes its kDim partials, so nothing in the scratch
  // needs clearing; the reduction reads exactly those entries.
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
  ALGX_CUDA(launch_dependent(qknorm_dgain_reduce, kReduceBlocks, kReduceThreads, 0, st, partial, grid, dgain));
  ALGX_LAUNCHED("qknorm_dgain_reduce launch");
  return ALGX_OK;
}

}  // extern "C"
