// Row RMS norm of any width and the SwiGLU gate, the two memory-bound
// elementwise families of the training step around the hot kernels
// (model.py:184-200): the ln1 / ln2 / embed / final norms (algebraic.py:76-83
// through model.py:158-159) and gate * silu(up) (model.py:193-198,
// standard.py:12-13).
//
// RMS norm: one warp per row, 128-bit loads, C 16-byte chunks per lane, the
// row's sum of squares by warp shuffles. The backward writes one fp32 row of
// dgain partials per CTA into the caller's workspace and a second launch sums
// them in a fixed order (deterministic for a given grid).
//
// SwiGLU: the gate and up projections come out of one GEMM as rows of
// [gate (f) | up (f)]; the forward reads both halves and writes y (rows, f),
// the backward reads the pair and dy and writes [dgate | dup]. Everything in
// fp32 between one bf16 load and one bf16 store per output, which is how XLA
// evaluates the fused bf16 chain (excess precision) in the reference.
#include <algorithm>

#include "algx_common.cuh"
#include "vec_io.cuh"

namespace algx {
namespace {

constexpr int kNormThreads = 256;  // 8 warps: one row per warp per pass
constexpr int kNormWarps = kNormThreads / 32;
constexpr int kNormMaxBlocks = 148 * 3;

// Forward: two rows per warp in flight (both rows' loads issued before
// either is used), the gain in shared memory.
// ADD: the row is s = x + r rounded to T (the residual add before the norm,
// model.py:180-200), written to s_out, then normalised.
template <typename T, int C, bool ADD>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(const T* __restrict__ x,
                                                                   const float* __restrict__ gain,
                                                                   T* __restrict__ y, int64_t rows, int dim,
                                                                   float eps, const T* __restrict__ r,
                                                                   T* __restrict__ s_out) {
  using V = Vec<T>;
  // gain, transposed to [element i of a chunk][chunk]: the lanes of a warp read
  // consecutive words (no bank conflicts)
  extern __shared__ float sg[];
  constexpr int CP = 32 * C;
  const int lane = threadIdx.x & 31;
  const int chunks = dim / V::N;
  for (int j = threadIdx.x; j < V::N * CP; j += kNormThreads) {
    const int i = j / CP, idx = j - i * CP;
    sg[j] = idx < chunks ? (gain ? gain[idx * V::N + i] : 1.f) : 0.f;
  }
  __syncthreads();
  const int64_t warps = (int64_t)gridDim.x * kNormWarps;
  for (int64_t r0 = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5); r0 < rows; r0 += 2 * warps) {
    uint4 raw[2][C];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t row = r0 + k * warps;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int idx = lane + 32 * c;
        raw[k][c] = (idx < chunks && row < rows) ? ld_stream(x + row * dim + idx * V::N) : make_uint4(0, 0, 0, 0);
      }
    }
    if constexpr (ADD) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t row = r0 + k * warps;
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const int idx = lane + 32 * c;
          const uint4 rr =
              (idx < chunks && row < rows) ? ld_stream(r + row * dim + idx * V::N) : make_uint4(0, 0, 0, 0);
          float a[V::N], b[V::N];
          unpack<T>(raw[k][c], a);
          unpack<T>(rr, b);
#pragma unroll
          for (int i = 0; i < V::N; ++i) a[i] += b[i];
          raw[k][c] = pack<T>(a);  // s = round(x + r)
          if (idx < chunks && row < rows) *reinterpret_cast<uint4*>(s_out + row * dim + idx * V::N) = raw[k][c];
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int64_t row = r0 + k * warps;
      float ss = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        float v[V::N];
        unpack<T>(raw[k][c], v);
#pragma unroll
        for (int i = 0; i < V::N; ++i) ss = fmaf(v[i], v[i], ss);
      }
      ss = row_sum<32>(ss);
      // mean = sum / dim, as jnp.mean divides (algebraic.py:79)
      const float tau = rsqrtf(ss / (float)dim + eps);
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int idx = lane + 32 * c;
        float v[V::N], o[V::N];
        unpack<T>(raw[k][c], v);
#pragma unroll
        for (int i = 0; i < V::N; ++i) o[i] = gain ? (v[i] * tau) * sg[i * CP + idx] : v[i] * tau;
        if (idx < chunks && row < rows) *reinterpret_cast<uint4*>(y + row * dim + idx * V::N) = pack<T>(o);
      }
    }
  }
}

// dx = tau (g dy) - x tau^3 mean(x g dy) (AD of the forward, the operation
// order of kernels/qk_norm.py:39-40); dgain partials = sum_rows dy (x tau).
// Two rows per warp are in flight (their loads issued before either is
// used); rows stay packed in registers, and the gain and the dgain
// accumulator sit in shared memory, so two CTAs fit on an SM.
constexpr int kNormBwdRows = 2;
constexpr int kNormBwdBlocks = 148 * 2;

// ADD: dx = round(norm backward + ds), ds the gradient that reaches the
// residual sum directly (the add's other consumer), in one rounding.
template <typename T, int C, bool ADD>
__global__ void __launch_bounds__(kNormThreads, 2) rmsnorm_bwd_kernel(const T* __restrict__ x,
                                                                      const float* __restrict__ gain,
                                                                      const T* __restrict__ dy, T* __restrict__ dx,
                                                                      float* __restrict__ partial, int64_t rows,
                                                                      int dim, float eps, const T* __restrict__ ds) {
  using V = Vec<T>;
  // Shared memory, all in the transposed [element i of a chunk][chunk] layout
  // so that the lanes of a warp touch consecutive words: each warp's dgain
  // accumulator [kNormWarps][N][32C], then the gain [N][32C].
  extern __shared__ float red[];
  constexpr int CP = 32 * C;
  constexpr int WS = V::N * CP;                  // floats per warp accumulator
  constexpr int R = (C <= 3 && !ADD) ? kNormBwdRows : 1;  // rows in flight per warp (else one, no spills)
  float* sg = red + kNormWarps * WS;
  float* acc = red + (threadIdx.x >> 5) * WS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int chunks = dim / V::N;
  for (int j = threadIdx.x; j < WS; j += kNormThreads) {
    const int i = j / CP, idx = j - i * CP;
    sg[j] = idx < chunks ? (gain ? gain[idx * V::N + i] : 1.f) : 0.f;
  }
  for (int j = threadIdx.x; j < kNormWarps * WS; j += kNormThreads) red[j] = 0.f;
  __syncthreads();
  const int64_t warps = (int64_t)gridDim.x * kNormWarps;
  for (int64_t r0 = (int64_t)blockIdx.x * kNormWarps + warp; r0 < rows; r0 += R * warps) {
    uint4 rx[R][C], rd[R][C];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int64_t row = r0 + k * warps;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int idx = lane + 32 * c;
        const bool ok = idx < chunks && row < rows;
        rx[k][c] = ok ? ld_stream(x + row * dim + idx * V::N) : make_uint4(0, 0, 0, 0);
        rd[k][c] = ok ? ld_stream(dy + row * dim + idx * V::N) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int64_t row = r0 + k * warps;
      float ss = 0.f, sdg = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int idx = lane + 32 * c;
        float xv[V::N], dv[V::N];
        unpack<T>(rx[k][c], xv);
        unpack<T>(rd[k][c], dv);
#pragma unroll
        for (int i = 0; i < V::N; ++i) {
          ss = fmaf(xv[i], xv[i], ss);
          sdg = fmaf(dv[i] * sg[i * CP + idx], xv[i], sdg);
        }
      }
      ss = row_sum<32>(ss);
      sdg = row_sum<32>(sdg);
      const float tau = rsqrtf(ss / (float)dim + eps);
      const float corr = tau * tau * tau * (sdg / (float)dim);
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int idx = lane + 32 * c;
        float xv[V::N], dv[V::N], o[V::N];
        unpack<T>(rx[k][c], xv);
        unpack<T>(rd[k][c], dv);
#pragma unroll
        for (int i = 0; i < V::N; ++i) {
          o[i] = (dv[i] * sg[i * CP + idx]) * tau - xv[i] * corr;
          acc[i * CP + idx] = fmaf(dv[i], xv[i] * tau, acc[i * CP + idx]);
        }
        if constexpr (ADD) {
          float dsv[V::N];
          unpack<T>((idx < chunks && row < rows) ? ld_stream(ds + row * dim + idx * V::N) : make_uint4(0, 0, 0, 0),
                    dsv);
#pragma unroll
          for (int i = 0; i < V::N; ++i) o[i] += dsv[i];
        }
        if (idx < chunks && row < rows) *reinterpret_cast<uint4*>(dx + row * dim + idx * V::N) = pack<T>(o);
      }
    }
  }
  if (!partial) return;  // no gain: no dgain
  __syncthreads();
  for (int col = threadIdx.x; col < dim; col += kNormThreads) {
    const int idx = col / V::N, i = col - idx * V::N;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kNormWarps; ++w) s += red[w * WS + i * CP + idx];
    partial[(int64_t)blockIdx.x * dim + col] = s;
  }
}

// dgain[col] = sum over the nb partial rows, in a fixed order: warp w sums rows
// w, w + 8, ... of 32 columns in four interleaved accumulators (so four loads
// are in flight), added in a fixed order; the 8 warp sums in warp order.
__global__ void __launch_bounds__(256) rmsnorm_dgain_reduce(const float* __restrict__ partial, int nb, int dim,
                                                           float* __restrict__ dgain) {
  __shared__ float red[8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  if (col < dim) {
    int b = warp;
    for (; b + 24 < nb; b += 32) {
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j] += partial[(int64_t)(b + 8 * j) * dim + col];
    }
    for (int j = 0; b < nb; b += 8, ++j) s[j & 3] += partial[(int64_t)b * dim + col];
  }
  red[warp][lane] = (s[0] + s[1]) + (s[2] + s[3]);
  __syncthreads();
  if (warp == 0 && col < dim) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][lane];
    dgain[col] = t;
  }
}

int norm_chunks(int64_t dim, int32_t dtype) {
  const int n = dtype == ALGX_BF16 ? 8 : 4;
  const int64_t per_lane = (dim / n + 31) / 32;
  // instantiated chunk counts per lane: dim <= 4096 (bf16), 2048 (float32)
  static const int kC[] = {1, 2, 3, 4, 6, 8, 12, 16};
  for (int c : kC)
    if (per_lane <= c) return c;
  return -1;
}

// Forward: one wave at three CTAs per SM (80 registers a thread at d = 768),
// two rows per warp per pass.
int norm_grid(int64_t rows) {
  int64_t g = (rows + 2 * kNormWarps - 1) / (2 * kNormWarps);
  if (g > kNormMaxBlocks) g = kNormMaxBlocks;
  return (int)(g < 1 ? 1 : g);
}

// One wave at two CTAs per SM; every warp keeps two rows in flight.
int norm_bwd_grid(int64_t rows) {
  int64_t g = (rows + kNormWarps * kNormBwdRows - 1) / (kNormWarps * kNormBwdRows);
  if (g > kNormBwdBlocks) g = kNormBwdBlocks;
  return (int)(g < 1 ? 1 : g);
}

// Pointers may be NULL only when there are no rows (empty tensors).
int check_norm(const void* x, const void* y, int64_t rows, int64_t dim, int32_t dtype, float eps, const char* who) {
  ALGX_REQUIRE(rows >= 0, std::string(who) + ": negative row count");
  ALGX_REQUIRE(rows == 0 || (x && y), std::string(who) + ": NULL pointer");
  ALGX_REQUIRE(dtype == ALGX_F32 || dtype == ALGX_BF16, std::string(who) + ": dtype must be float32 or bfloat16");
  ALGX_REQUIRE(eps > 0.f, std::string(who) + ": epsilon must be positive");
  const int n = dtype == ALGX_BF16 ? 8 : 4;
  ALGX_REQUIRE(dim > 0 && dim % n == 0, std::string(who) + ": width must be a positive multiple of 16 bytes");
  ALGX_REQUIRE(norm_chunks(dim, dtype) > 0,
               std::string(who) + ": width above the supported maximum (4096 bf16, 2048 float32)");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0,
               std::string(who) + ": tensors must be 16-byte aligned");
  return ALGX_OK;
}

template <typename T, int C>
void launch_norm_fwd(const void* x, const float* gain, void* y, int64_t rows, int dim, float eps, cudaStream_t st,
                     const void* r, void* s_out) {
  // the transposed gain: N x 32C floats (at most 16 KB)
  const size_t smem = (size_t)Vec<T>::N * 32 * C * sizeof(float);
  if (r)
    rmsnorm_fwd_kernel<T, C, true><<<norm_grid(rows), kNormThreads, smem, st>>>(
        static_cast<const T*>(x), gain, static_cast<T*>(y), rows, dim, eps, static_cast<const T*>(r),
        static_cast<T*>(s_out));
  else
    rmsnorm_fwd_kernel<T, C, false><<<norm_grid(rows), kNormThreads, smem, st>>>(
        static_cast<const T*>(x), gain, static_cast<T*>(y), rows, dim, eps, nullptr, nullptr);
}

template <typename T, int C>
cudaError_t launch_norm_bwd(const void* x, const float* gain, const void* dy, void* dx, float* partial,
                            int64_t rows, int dim, float eps, cudaStream_t st, const void* ds) {
  const size_t smem = (size_t)(kNormWarps + 1) * Vec<T>::N * 32 * C * sizeof(float);
  auto kern = ds ? rmsnorm_bwd_kernel<T, C, true> : rmsnorm_bwd_kernel<T, C, false>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kern<<<norm_bwd_grid(rows), kNormThreads, smem, st>>>(static_cast<const T*>(x), gain, static_cast<const T*>(dy),
                                                        static_cast<T*>(dx), partial, rows, dim, eps,
                                                        static_cast<const T*>(ds));
  return cudaSuccess;
}

template <typename T>
void dispatch_norm_fwd(int C, const void* x, const float* gain, void* y, int64_t rows, int dim, float eps,
                       cudaStream_t st, const void* r = nullptr, void* s_out = nullptr) {
  switch (C) {
    case 1: launch_norm_fwd<T, 1>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    case 2: launch_norm_fwd<T, 2>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    case 3: launch_norm_fwd<T, 3>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    case 4: launch_norm_fwd<T, 4>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    case 6: launch_norm_fwd<T, 6>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    case 8: launch_norm_fwd<T, 8>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    case 12: launch_norm_fwd<T, 12>(x, gain, y, rows, dim, eps, st, r, s_out); break;
    default: launch_norm_fwd<T, 16>(x, gain, y, rows, dim, eps, st, r, s_out); break;
  }
}

template <typename T>
cudaError_t dispatch_norm_bwd(int C, const void* x, const float* gain, const void* dy, void* dx, float* partial,
                              int64_t rows, int dim, float eps, cudaStream_t st, const void* ds = nullptr) {
  switch (C) {
    case 1: return launch_norm_bwd<T, 1>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    case 2: return launch_norm_bwd<T, 2>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    case 3: return launch_norm_bwd<T, 3>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    case 4: return launch_norm_bwd<T, 4>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    case 6: return launch_norm_bwd<T, 6>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    case 8: return launch_norm_bwd<T, 8>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    case 12: return launch_norm_bwd<T, 12>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
    default: return launch_norm_bwd<T, 16>(x, gain, dy, dx, partial, rows, dim, eps, st, ds);
  }
}

// ------------------------------------------------------------------ SwiGLU
constexpr int kGluThreads = 256;
constexpr int kGluMaxBlocks = 148 * 8;

__device__ __forceinline__ float sigmoid_f(float u) { return 1.f / (1.f + __expf(-u)); }

// y[r, j] = gate[r, j] * up[r, j] * sigmoid(up[r, j]), gu[r] = [gate | up]
__global__ void __launch_bounds__(kGluThreads) swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                                                 __nv_bfloat16* __restrict__ y, int64_t rows,
                                                                 int ff) {
  const int cpr = ff / 8;  // 16-byte chunks per output row
  const int64_t total = rows * cpr;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kGluThreads) {
    const int64_t r = i / cpr;
    const int c = (int)(i - r * cpr);
    const __nv_bfloat16* src = gu + r * 2 * ff + c * 8;
    float g[8], u[8], o[8];
    unpack<__nv_bfloat16>(ld_stream(src), g);
    unpack<__nv_bfloat16>(ld_stream(src + ff), u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = g[k] * (u[k] * sigmoid_f(u[k]));
    *reinterpret_cast<uint4*>(y + r * ff + c * 8) = pack<__nv_bfloat16>(o);
  }
}

// dgate = dy silu(up); dup = dy gate (s + up s (1 - s)), s = sigmoid(up)
__global__ void __launch_bounds__(kGluThreads) swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                                                 const __nv_bfloat16* __restrict__ dy,
                                                                 __nv_bfloat16* __restrict__ dgu, int64_t rows,
                                                                 int ff) {
  const int cpr = ff / 8;
  const int64_t total = rows * cpr;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kGluThreads) {
    const int64_t r = i / cpr;
    const int c = (int)(i - r * cpr);
    const __nv_bfloat16* src = gu + r * 2 * ff + c * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    unpack<__nv_bfloat16>(ld_stream(src), g);
    unpack<__nv_bfloat16>(ld_stream(src + ff), u);
    unpack<__nv_bfloat16>(ld_stream(dy + r * ff + c * 8), d);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = sigmoid_f(u[k]);
      dg[k] = d[k] * (u[k] * s);
      du[k] = (d[k] * g[k]) * (s + u[k] * s * (1.f - s));
    }
    __nv_bfloat16* dst = dgu + r * 2 * ff + c * 8;
    *reinterpret_cast<uint4*>(dst) = pack<__nv_bfloat16>(dg);
    *reinterpret_cast<uint4*>(dst + ff) = pack<__nv_bfloat16>(du);
  }
}

// ALU-GLU (algebraic.py:86-117, model.py:196-197): act = alu(up, beta)
// rounded to bf16 (_alu_parts' astype), y = bf16(gate * act). alu(z) =
// z/2 (1 + u), u = bz / sqrt(1 + b^2 z^2); for bz < 0 the factor 1 + u is
// formed as r^2 / (1 - u) so the negative tail keeps its precision.
__device__ __forceinline__ void alu_parts(float z, float beta, float& act, float& u, float& r) {
  const float bz = beta * z;
  r = rsqrtf(1.f + bz * bz);
  u = bz * r;
  const float opu = bz < 0.f ? (r * r) / (1.f - u) : 1.f + u;
  act = round_io<__nv_bfloat16>(0.5f * z * opu);
}

__global__ void __launch_bounds__(kGluThreads) aluglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                                                 __nv_bfloat16* __restrict__ y, int64_t rows, int ff,
                                                                 float beta) {
  const int cpr = ff / 8;
  const int64_t total = rows * cpr;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kGluThreads) {
    const int64_t r = i / cpr;
    const int c = (int)(i - r * cpr);
    const __nv_bfloat16* src = gu + r * 2 * ff + c * 8;
    float g[8], z[8], o[8];
    unpack<__nv_bfloat16>(ld_stream(src), g);
    unpack<__nv_bfloat16>(ld_stream(src + ff), z);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float act, u, rr;
      alu_parts(z[k], beta, act, u, rr);
      o[k] = g[k] * act;
    }
    *reinterpret_cast<uint4*>(y + r * ff + c * 8) = pack<__nv_bfloat16>(o);
  }
}

// The reference's custom VJP (algebraic.py:109-113): the cotangent of act is
// bf16(dy * gate); dup = bf16(g * (0.5 (1 + u) + 0.5 u r^2)); dgate = bf16(dy * act).
__global__ void __launch_bounds__(kGluThreads) aluglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                                                 const __nv_bfloat16* __restrict__ dy,
                                                                 __nv_bfloat16* __restrict__ dgu, int64_t rows,
                                                                 int ff, float beta) {
  const int cpr = ff / 8;
  const int64_t total = rows * cpr;
  for (int64_t i = (int64_t)blockIdx.x * kGluThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kGluThreads) {
    const int64_t r = i / cpr;
    const int c = (int)(i - r * cpr);
    const __nv_bfloat16* src = gu + r * 2 * ff + c * 8;
    float g[8], z[8], d[8], dg[8], dz[8];
    unpack<__nv_bfloat16>(ld_stream(src), g);
    unpack<__nv_bfloat16>(ld_stream(src + ff), z);
    unpack<__nv_bfloat16>(ld_stream(dy + r * ff + c * 8), d);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float act, u, rr;
      alu_parts(z[k], beta, act, u, rr);
      const float gact = round_io<__nv_bfloat16>(d[k] * g[k]);
      const float deriv = 0.5f * (1.f + u) + 0.5f * u * (rr * rr);
      dg[k] = d[k] * act;
      dz[k] = gact * deriv;
    }
    __nv_bfloat16* dst = dgu + r * 2 * ff + c * 8;
    *reinterpret_cast<uint4*>(dst) = pack<__nv_bfloat16>(dg);
    *reinterpret_cast<uint4*>(dst + ff) = pack<__nv_bfloat16>(dz);
  }
}

int glu_grid(int64_t rows, int64_t ff) {
  const int64_t total = rows * (ff / 8);
  int64_t g = (total + kGluThreads - 1) / kGluThreads;
  if (g > kGluMaxBlocks) g = kGluMaxBlocks;
  return (int)(g < 1 ? 1 : g);
}

int check_glu(const void* a, const void* b, int64_t rows, int64_t ff, const char* who) {
  ALGX_REQUIRE(rows >= 0, std::string(who) + ": negative row count");
  ALGX_REQUIRE(rows == 0 || (a && b), std::string(who) + ": NULL pointer");
  ALGX_REQUIRE(ff > 0 && ff % 8 == 0, std::string(who) + ": hidden width must be a positive multiple of 8");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0,
               std::string(who) + ": tensors must be 16-byte aligned");
  return ALGX_OK;
}

// ------------------------------------------------------- head/token order
// Attention tensors are head-major (B, H, T, 64) for the TMA-fed kernels;
// the model's projections produce and consume token-major (B, T, H, 64).
// One 64-element row moves per TPR threads with 16-byte accesses; the rows
// are read in one order and written in the other.
constexpr int kPermThreads = 256;
constexpr int kPermUnroll = 4;

template <typename T>
__global__ void __launch_bounds__(kPermThreads) permute_rows_kernel(const T* __restrict__ src, T* __restrict__ dst,
                                                                   int64_t rows, int T_, int H, int to_tokens) {
  using V = Vec<T>;
  const int lane = threadIdx.x & 31, sub = lane % V::TPR, rl = lane / V::TPR;
  const int64_t warps = (int64_t)gridDim.x * (kPermThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kPermThreads / 32) + (threadIdx.x >> 5);
  for (int64_t r0 = w * V::RPW * kPermUnroll; r0 < rows; r0 += warps * V::RPW * kPermUnroll) {
    uint4 raw[kPermUnroll];
    int64_t other[kPermUnroll];
#pragma unroll
    for (int u = 0; u < kPermUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;  // head-major index (b*H + h)*T + t, below 2^31
      const unsigned r = (unsigned)row, bh = r / (unsigned)T_, t = r - bh * (unsigned)T_;
      const unsigned b = bh / (unsigned)H, h = bh - b * (unsigned)H;
      other[u] = ((int64_t)b * T_ + t) * H + h;  // token-major index
      const int64_t from = to_tokens ? row : other[u];
      raw[u] = row < rows ? ld_stream(src + from * kRowDim + sub * V::N) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kPermUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      const int64_t to = to_tokens ? other[u] : row;
      if (row < rows) *reinterpret_cast<uint4*>(dst + to * kRowDim + sub * V::N) = raw[u];
    }
  }
}

int permute_rows(const void* src, void* dst, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                 int to_tokens, void* stream, const char* who) {
  ALGX_REQUIRE(B >= 0 && H > 0 && T > 0 && D == kRowDim, std::string(who) + ": needs D = 64 and positive H, T");
  ALGX_REQUIRE(dtype == ALGX_F32 || dtype == ALGX_BF16, std::string(who) + ": dtype must be float32 or bfloat16");
  const int64_t rows = B * H * T;
  if (rows == 0) return ALGX_OK;
  ALGX_REQUIRE(src && dst && src != dst, std::string(who) + ": NULL or aliased pointers");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
               std::string(who) + ": tensors must be 16-byte aligned");
  ALGX_REQUIRE(rows <= INT32_MAX, std::string(who) + ": B*H*T must be below 2^31");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rpw = dtype == ALGX_BF16 ? Vec<__nv_bfloat16>::RPW : Vec<float>::RPW;
  const int64_t per_block = (int64_t)(kPermThreads / 32) * rpw * kPermUnroll;
  const int grid = (int)std::min<int64_t>((rows + per_block - 1) / per_block, 148 * 8);
  if (dtype == ALGX_BF16)
    permute_rows_kernel<__nv_bfloat16><<<grid, kPermThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), rows, (int)T, (int)H, to_tokens);
  else
    permute_rows_kernel<float><<<grid, kPermThreads, 0, st>>>(static_cast<const float*>(src), static_cast<float*>(dst),
                                                              rows, (int)T, (int)H, to_tokens);
  ALGX_LAUNCHED("permute_rows launch");
  return ALGX_OK;
}

}  // namespace
}  // namespace algx

using namespace algx;

extern "C" {

int algx_rmsnorm_fwd(const void* x, const float* gain, void* y, int64_t rows, int64_t dim, int32_t dtype, float eps,
                     void* stream) {
  if (int s = check_norm(x, y, rows, dim, dtype, eps, "rmsnorm_fwd")) return s;
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int C = norm_chunks(dim, dtype);
  if (dtype == ALGX_BF16)
    dispatch_norm_fwd<__nv_bfloat16>(C, x, gain, y, rows, (int)dim, eps, st);
  else
    dispatch_norm_fwd<float>(C, x, gain, y, rows, (int)dim, eps, st);
  ALGX_LAUNCHED("rmsnorm_fwd launch");
  return ALGX_OK;
}

size_t algx_rmsnorm_bwd_workspace_size(int64_t rows, int64_t dim) {
  if (rows <= 0 || dim <= 0) return 0;
  return (size_t)norm_bwd_grid(rows) * (size_t)dim * sizeof(float);
}

int algx_rmsnorm_bwd(const void* x, const float* gain, const void* dy, void* dx, float* dgain, int64_t rows,
                     int64_t dim, int32_t dtype, float eps, void* workspace, size_t workspace_bytes, void* stream) {
  if (int s = check_norm(x, dx, rows, dim, dtype, eps, "rmsnorm_bwd")) return s;
  ALGX_REQUIRE(rows == 0 || dy, "rmsnorm_bwd: NULL pointer");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(dy) & 15) == 0, "rmsnorm_bwd: tensors must be 16-byte aligned");
  ALGX_REQUIRE(!gain || dgain, "rmsnorm_bwd: a gain needs a dgain output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (gain) ALGX_CUDA(cudaMemsetAsync(dgain, 0, (size_t)dim * sizeof(float), st));
    return ALGX_OK;
  }
  const int grid = norm_bwd_grid(rows);
  float* partial = nullptr;
  if (gain) {
    ALGX_REQUIRE(workspace && workspace_bytes >= (size_t)grid * (size_t)dim * sizeof(float),
                 "rmsnorm_bwd: workspace too small (see algx_rmsnorm_bwd_workspace_size)");
    partial = static_cast<float*>(workspace);
  }
  const int C = norm_chunks(dim, dtype);
  if (dtype == ALGX_BF16)
    ALGX_CUDA(dispatch_norm_bwd<__nv_bfloat16>(C, x, gain, dy, dx, partial, rows, (int)dim, eps, st));
  else
    ALGX_CUDA(dispatch_norm_bwd<float>(C, x, gain, dy, dx, partial, rows, (int)dim, eps, st));
  ALGX_LAUNCHED("rmsnorm_bwd launch");
  if (gain) {
    rmsnorm_dgain_reduce<<<(unsigned)((dim + 31) / 32), 256, 0, st>>>(partial, grid, (int)dim, dgain);
    ALGX_LAUNCHED("rmsnorm_dgain_reduce launch");
  }
  return ALGX_OK;
}

int algx_add_rmsnorm_fwd(const void* x, const void* r, const float* gain, void* s_out, void* y, int64_t rows,
                         int64_t dim, int32_t dtype, float eps, void* stream) {
  if (int st = check_norm(x, y, rows, dim, dtype, eps, "add_rmsnorm_fwd")) return st;
  ALGX_REQUIRE(rows == 0 || (r && s_out), "add_rmsnorm_fwd: NULL pointer");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(r) & 15) == 0 && (reinterpret_cast<uintptr_t>(s_out) & 15) == 0,
               "add_rmsnorm_fwd: tensors must be 16-byte aligned");
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int C = norm_chunks(dim, dtype);
  if (dtype == ALGX_BF16)
    dispatch_norm_fwd<__nv_bfloat16>(C, x, gain, y, rows, (int)dim, eps, st, r, s_out);
  else
    dispatch_norm_fwd<float>(C, x, gain, y, rows, (int)dim, eps, st, r, s_out);
  ALGX_LAUNCHED("add_rmsnorm_fwd launch");
  return ALGX_OK;
}

int algx_add_rmsnorm_bwd(const void* s, const float* gain, const void* dy, const void* ds, void* dx, float* dgain,
                         int64_t rows, int64_t dim, int32_t dtype, float eps, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (int st = check_norm(s, dx, rows, dim, dtype, eps, "add_rmsnorm_bwd")) return st;
  ALGX_REQUIRE(rows == 0 || (dy && ds), "add_rmsnorm_bwd: NULL pointer");
  ALGX_REQUIRE((reinterpret_cast<uintptr_t>(dy) & 15) == 0 && (reinterpret_cast<uintptr_t>(ds) & 15) == 0,
               "add_rmsnorm_bwd: tensors must be 16-byte aligned");
  ALGX_REQUIRE(!gain || dgain, "add_rmsnorm_bwd: a gain needs a dgain output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (gain) ALGX_CUDA(cudaMemsetAsync(dgain, 0, (size_t)dim * sizeof(float), st));
    return ALGX_OK;
  }
  const int grid = norm_bwd_grid(rows);
  float* partial = nullptr;
  if (gain) {
    ALGX_REQUIRE(workspace && workspace_bytes >= (size_t)grid * (size_t)dim * sizeof(float),
                 "add_rmsnorm_bwd: workspace too small (see algx_rmsnorm_bwd_workspace_size)");
    partial = static_cast<float*>(workspace);
  }
  const int C = norm_chunks(dim, dtype);
  if (dtype == ALGX_BF16)
    ALGX_CUDA(dispatch_norm_bwd<__nv_bfloat16>(C, s, gain, dy, dx, partial, rows, (int)dim, eps, st, ds));
  else
    ALGX_CUDA(dispatch_norm_bwd<float>(C, s, gain, dy, dx, partial, rows, (int)dim, eps, st, ds));
  ALGX_LAUNCHED("add_rmsnorm_bwd launch");
  if (gain) {
    rmsnorm_dgain_reduce<<<(unsigned)((dim + 31) / 32), 256, 0, st>>>(partial, grid, (int)dim, dgain);
    ALGX_LAUNCHED("rmsnorm_dgain_reduce launch");
  }
  return ALGX_OK;
}

int algx_swiglu_fwd(const void* gu, void* y, int64_t rows, int64_t ff, void* stream) {
  if (int s = check_glu(gu, y, rows, ff, "swiglu_fwd")) return s;
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  swiglu_fwd_kernel<<<glu_grid(rows, ff), kGluThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(gu),
                                                                static_cast<__nv_bfloat16*>(y), rows, (int)ff);
  ALGX_LAUNCHED("swiglu_fwd launch");
  return ALGX_OK;
}

int algx_swiglu_bwd(const void* gu, const void* dy, void* dgu, int64_t rows, int64_t ff, void* stream) {
  if (int s = check_glu(gu, dgu, rows, ff, "swiglu_bwd")) return s;
  ALGX_REQUIRE((rows == 0 || dy) && (reinterpret_cast<uintptr_t>(dy) & 15) == 0,
               "swiglu_bwd: dy NULL or not 16-byte aligned");
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  swiglu_bwd_kernel<<<glu_grid(rows, ff), kGluThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(gu),
                                                                static_cast<const __nv_bfloat16*>(dy),
                                                                static_cast<__nv_bfloat16*>(dgu), rows, (int)ff);
  ALGX_LAUNCHED("swiglu_bwd launch");
  return ALGX_OK;
}

int algx_aluglu_fwd(const void* gu, void* y, int64_t rows, int64_t ff, float beta, void* stream) {
  if (int s = check_glu(gu, y, rows, ff, "aluglu_fwd")) return s;
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  aluglu_fwd_kernel<<<glu_grid(rows, ff), kGluThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(gu),
                                                                static_cast<__nv_bfloat16*>(y), rows, (int)ff, beta);
  ALGX_LAUNCHED("aluglu_fwd launch");
  return ALGX_OK;
}

int algx_aluglu_bwd(const void* gu, const void* dy, void* dgu, int64_t rows, int64_t ff, float beta, void* stream) {
  if (int s = check_glu(gu, dgu, rows, ff, "aluglu_bwd")) return s;
  ALGX_REQUIRE((rows == 0 || dy) && (reinterpret_cast<uintptr_t>(dy) & 15) == 0,
               "aluglu_bwd: dy NULL or not 16-byte aligned");
  if (rows == 0) return ALGX_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  aluglu_bwd_kernel<<<glu_grid(rows, ff), kGluThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(gu),
                                                                static_cast<const __nv_bfloat16*>(dy),
                                                                static_cast<__nv_bfloat16*>(dgu), rows, (int)ff, beta);
  ALGX_LAUNCHED("aluglu_bwd launch");
  return ALGX_OK;
}

int algx_heads_to_tokens(const void* src, void* dst, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                         void* stream) {
  return permute_rows(src, dst, B, H, T, D, dtype, 1, stream, "heads_to_tokens");
}

int algx_tokens_to_heads(const void* src, void* dst, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                         void* stream) {
  return permute_rows(src, dst, B, H, T, D, dtype, 0, stream, "tokens_to_heads");
}

}  // extern "C"
