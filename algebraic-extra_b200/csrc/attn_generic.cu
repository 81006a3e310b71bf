// Attention: scale fold + range guard (prepare), the generic CUDA-core
// forward/backward for every variant and I/O dtype, the di / sink-gradient
// reductions, and the C-ABI entry points that dispatch between these and the
// tcgen05 fast path (attn_tc.cu).
//
// The generic kernels restate kernels/flash.py:189-284 (forward) and
// :333-361 (_tile_grads) one query row (or key row) per thread, with the
// reference's rounding points: p is rounded to the value dtype before P.V
// and dV, ds to the query dtype before dK/dQ, o to the query dtype. They
// serve fp32 I/O, the shifted/softmax branches and shapes the fast path
// does not take.
#include <algorithm>

#include <type_traits>

#include "attn_common.cuh"
#include "attn_tc.h"
#include "tmap.h"
#include "vec_io.cuh"

namespace algx {
namespace {

constexpr int kD = 64;
constexpr int kRows = 128;  // query (or key) rows per CTA, one per thread
constexpr int kKT = 32;     // keys (or queries) per shared-memory tile
constexpr int kPrepThreads = 256;

// ------------------------------------------------------------------ prepare
template <typename T>
__global__ void __launch_bounds__(kPrepThreads) attn_prepare_kernel(const T* __restrict__ q,
                                                                    const T* __restrict__ k,
                                                                    const T* __restrict__ v,
                                                                    const float* __restrict__ sink, int H,
                                                                    T* __restrict__ qs, float* guard,
                                                                    int64_t rows, float scale) {
  using V = Vec<T>;
  const int which = blockIdx.y;  // 0: q (scaled, written), 1: k, 2: v
  const T* src = which == 0 ? q : (which == 1 ? k : v);
  const int lane = threadIdx.x & 31;
  const int sub = lane % V::TPR;
  const int rl = lane / V::TPR;
  const int64_t warps = (int64_t)gridDim.x * (kPrepThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kPrepThreads / 32) + (threadIdx.x >> 5);
  float local = 0.f;
  for (int64_t r0 = w * V::RPW; r0 < rows; r0 += warps * V::RPW) {
    const int64_t row = r0 + rl;
    const bool ok = row < rows;
    float x[V::N];
    uint4 raw = ok ? ld_stream(src + row * kD + sub * V::N) : make_uint4(0, 0, 0, 0);
    unpack<T>(raw, x);
    if (which == 2) {
#pragma unroll
      for (int i = 0; i < V::N; ++i) local = nan_max(local, fabsf(x[i]));
    } else {
      if (which == 0) {
#pragma unroll
        for (int i = 0; i < V::N; ++i) x[i] = round_io<T>(x[i] * scale);
        if (ok) *reinterpret_cast<uint4*>(qs + row * kD + sub * V::N) = pack<T>(x);
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) ss = fmaf(x[i], x[i], ss);
      ss = row_sum<V::TPR>(ss);
      local = nan_max(local, ss);
    }
  }
  __shared__ float red[kPrepThreads / 32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local = nan_max(local, __shfl_xor_sync(0xffffffffu, local, off));
  if (lane == 0) red[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < kPrepThreads / 32; ++i) m = nan_max(m, red[i]);
    atomic_max_nonneg(&guard[which], __int_as_float(__float_as_int(m) & 0x7fffffff));
  }
  if (which == 0 && blockIdx.x == 0 && sink != nullptr) {
    for (int t = threadIdx.x; t < H; t += kPrepThreads) {
      const float a = fabsf(sink[t]);
      atomic_max_nonneg(&guard[3], __int_as_float(__float_as_int(a) & 0x7fffffff));
    }
  }
}

// Fused attention prologue (model.py:170-174 then flash.py:823-849): the QK
// RMS norm of q and k (qk_norm.py:29-43, algebraic.py:76-83) and the prepare
// step above in one pass over q, k and v. Each value goes through the same
// rounding points as the separate launches: y = bf16((x * tau) * gain), then
// q_scaled = bf16(y * scale); the guard maxima are taken over the rounded
// q_scaled and normalised k rows, and over v and the sink as in prepare.
// Rotate-half rotation of one D = 64 row by the (T, 32) tables cos, sin
// (algebraic.py:172-179): y1 = x1 c - x2 s, y2 = x1 s + x2 c, with the table
// entries rounded to the I/O dtype first and the products and sum taken in
// fp32 (no contraction), rounded once. INVERSE applies the transpose
// (dx1 = dy1 c + dy2 s, dx2 = dy2 c - dy1 s), the rotation's VJP. The thread
// holding elements j.. of one half swaps values with the thread holding j + 32
// of the other (lane ^ TPR/2), so every lane of the warp must call it.
template <typename T, bool INVERSE>
__device__ __forceinline__ void rotate_half(float (&x)[Vec<T>::N], const float* __restrict__ cosv,
                                            const float* __restrict__ sinv, int64_t t, int sub) {
  using V = Vec<T>;
  constexpr int kHalfT = V::TPR / 2;
  const bool first = sub < kHalfT;
  const int j0 = (sub % kHalfT) * V::N;
  const float* cr = cosv + t * (kD / 2) + j0;
  const float* sr = sinv + t * (kD / 2) + j0;
#pragma unroll
  for (int i = 0; i < V::N; ++i) {
    const float other = __shfl_xor_sync(0xffffffffu, x[i], kHalfT);
    const float c = round_io<T>(cr[i]), s = round_io<T>(sr[i]);
    const float own_c = __fmul_rn(x[i], c), other_s = __fmul_rn(other, s);
    const bool minus = INVERSE ? !first : first;  // own * c - other * s, else own * c + other * s
    x[i] = round_io<T>(minus ? __fsub_rn(own_c, other_s) : __fadd_rn(own_c, other_s));
  }
}

// Row of head-major index row = (b*H + h)*T + t in a token-major tensor whose
// rows (b, t) hold `stride` rows of 64 elements, head h at offset h (the
// caller offsets the base pointer to the q, k or v block). stride 0: the
// tensor is head-major itself.
// The packed entry points require B*H*T < 2^31, so the index splits use
// 32-bit division (a 64-bit division costs several times as many instructions,
// once per row and thread).
__device__ __forceinline__ int64_t tok_row(int64_t row, int T_, int H, int stride) {
  if (stride == 0) return row;
  const unsigned r = (unsigned)row;
  const unsigned bh = r / (unsigned)T_;
  const unsigned t = r - bh * (unsigned)T_;
  const unsigned b = bh / (unsigned)H;
  const unsigned h = bh - b * (unsigned)H;
  return ((int64_t)b * T_ + t) * stride + h;
}

// in_stride > 0: q, k, v are the blocks of one token-major (B, T, 3, H, D)
// tensor (row stride in_stride = 3H), and vh (when not NULL) receives v in
// head-major order for the TMA-fed attention kernels.
template <typename T, bool ROT, bool PACKED>
__global__ void __launch_bounds__(kPrepThreads) qknorm_attn_prepare_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ gain_q,
    const float* __restrict__ gain_k, const float* __restrict__ rot_cos, const float* __restrict__ rot_sin,
    const float* __restrict__ sink, int H, int T_, T* __restrict__ qs, T* __restrict__ kn, float* guard,
    int64_t rows, float scale, float eps, int in_stride, T* __restrict__ vh) {
  // No early griddepcontrol.launch_dependents: the forward, a programmatic
  // dependent, is scheduled when this multi-wave grid finishes, so its CTAs do
  // not take SMs this grid's later waves need.
  using V = Vec<T>;
  constexpr int kUnroll = 4;
  const int which = blockIdx.y;  // 0: q (normalised, scaled, written), 1: k (normalised, written), 2: v
  const T* src = which == 0 ? q : (which == 1 ? k : v);
  T* dst = which == 0 ? qs : kn;
  const float* gain = which == 0 ? gain_q : gain_k;
  const int lane = threadIdx.x & 31;
  const int sub = lane % V::TPR;
  const int rl = lane / V::TPR;
  float g[V::N];
#pragma unroll
  for (int i = 0; i < V::N; ++i) g[i] = which == 2 ? 0.f : gain[sub * V::N + i];
  const int64_t warps = (int64_t)gridDim.x * (kPrepThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kPrepThreads / 32) + (threadIdx.x >> 5);
  float local = 0.f;
  for (int64_t r0 = w * V::RPW * kUnroll; r0 < rows; r0 += warps * V::RPW * kUnroll) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      const int64_t srow = PACKED ? tok_row(row, T_, H, in_stride) : row;
      raw[u] = row < rows ? ld_stream(src + srow * kD + sub * V::N) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      const bool ok = row < rows;
      float x[V::N];
      unpack<T>(raw[u], x);
      if (which == 2) {
#pragma unroll
        for (int i = 0; i < V::N; ++i) local = nan_max(local, fabsf(x[i]));
        if constexpr (PACKED) {
          if (ok) *reinterpret_cast<uint4*>(vh + row * kD + sub * V::N) = raw[u];
        }
        continue;
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) ss = fmaf(x[i], x[i], ss);
      ss = row_sum<V::TPR>(ss);
      const float tau = rsqrtf(ss * (1.0f / kD) + eps);
#pragma unroll
      for (int i = 0; i < V::N; ++i) x[i] = round_io<T>((x[i] * tau) * g[i]);
      if constexpr (ROT) rotate_half<T, false>(x, rot_cos, rot_sin, row % T_, sub);
      if (which == 0) {
#pragma unroll
        for (int i = 0; i < V::N; ++i) x[i] = round_io<T>(x[i] * scale);
      }
      if (ok) *reinterpret_cast<uint4*>(dst + row * kD + sub * V::N) = pack<T>(x);
      float s2 = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) s2 = fmaf(x[i], x[i], s2);
      s2 = row_sum<V::TPR>(s2);
      local = nan_max(local, s2);
    }
  }
  __shared__ float red[kPrepThreads / 32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) local = nan_max(local, __shfl_xor_sync(0xffffffffu, local, off));
  if (lane == 0) red[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int i = 0; i < kPrepThreads / 32; ++i) m = nan_max(m, red[i]);
    atomic_max_nonneg(&guard[which], __int_as_float(__float_as_int(m) & 0x7fffffff));
  }
  if (which == 0 && blockIdx.x == 0 && sink != nullptr) {
    for (int t = threadIdx.x; t < H; t += kPrepThreads) {
      const float a = fabsf(sink[t]);
      atomic_max_nonneg(&guard[3], __int_as_float(__float_as_int(a) & 0x7fffffff));
    }
  }
}

// ------------------------------------------------------------------ forward
template <typename T>
__device__ __forceinline__ void attn_fwd_generic_tile(algx_attn_config cfg, const T* __restrict__ q,
                                                          const T* __restrict__ k, const T* __restrict__ v,
                                                          const float* __restrict__ sink,
                                                          const float* __restrict__ guard, T* __restrict__ o,
                                                          float* __restrict__ o_prec, float* __restrict__ stat,
                                                          int H, int T_, int blk_tile, int bh_tile, const Eff e) {
  __shared__ float ks[kKT][kD];
  __shared__ float vs[kKT][kD];
  const int bh = bh_tile;
  const int h = bh % H;
  const int row0 = blk_tile * kRows;
  const int row = row0 + threadIdx.x;
  const bool active = row < T_;
  const size_t base = (size_t)bh * T_ * kD;
  const int n = cfg.n;
  float qr[kD], acc[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) {
    qr[d] = active ? to_f32(q[base + (size_t)row * kD + d]) : 0.f;
    acc[d] = 0.f;
  }
  const bool hs = cfg.has_sink != 0;
  const float b = hs ? sink[h] : 0.f;
  float m = 0.f, l = 0.f, r;
  if (e.branch == BR_UNSHIFTED) {
    if (hs) l = ipow(rho_sel(e.clip ? fminf(b, cfg.clamp) : b, e.fast, r), n);
  } else if (hs) {
    m = b;
    l = 1.f;
  } else {
    m = -1e4f;
  }
  bool first = true;
  const int last = min(T_, row0 + kRows) - 1;
  const int ntiles = last / kKT + 1;
  for (int t = 0; t < ntiles; ++t) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKT * kD; i += kRows) {
      const int j = i / kD, d = i % kD, key = t * kKT + j;
      ks[j][d] = key < T_ ? to_f32(k[base + (size_t)key * kD + d]) : 0.f;
      vs[j][d] = key < T_ ? to_f32(v[base + (size_t)key * kD + d]) : 0.f;
    }
    __syncthreads();
    if (!active || t * kKT > row) continue;
    const int nvalid = min(kKT, row - t * kKT + 1);
    float s[kKT];
#pragma unroll
    for (int j = 0; j < kKT; ++j) {
      float a = 0.f;
#pragma unroll
      for (int d = 0; d < kD; ++d) a = fmaf(qr[d], ks[j][d], a);
      s[j] = a;
    }
    if (e.branch == BR_UNSHIFTED) {
#pragma unroll
      for (int j = 0; j < kKT; ++j) {
        if (j < nvalid) {
          const float x = e.clip ? fminf(s[j], cfg.clamp) : s[j];
          const float p = ipow(rho_sel(x, e.fast, r), n);
          l += p;
          const float pb = round_io<T>(p);
#pragma unroll
          for (int d = 0; d < kD; ++d) acc[d] = fmaf(pb, vs[j][d], acc[d]);
        }
      }
    } else {
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < kKT; ++j)
        if (j < nvalid) tmax = fmaxf(tmax, s[j]);
      float m_new = fmaxf(m, tmax), m_prev = m;
      if (!hs && first) {
        m_new = tmax;
        m_prev = m_new;
      }
      float alpha, shift = 1.f;
      if (e.branch == BR_SOFTMAX) {
        alpha = expf(m_prev - m_new);
      } else {
        shift = rho_exact(-m_new, r);
        alpha = ipow(rho_exact(m_prev, r) * shift, n);
      }
      l *= alpha;
#pragma unroll
      for (int d = 0; d < kD; ++d) acc[d] *= alpha;
#pragma unroll
      for (int j = 0; j < kKT; ++j) {
        if (j < nvalid) {
          const float p = e.branch == BR_SOFTMAX ? expf(s[j] - m_new)
                                                 : ipow(rho_sel(s[j], e.fast, r) * shift, n);
          l += p;
          const float pb = round_io<T>(p);
#pragma unroll
          for (int d = 0; d < kD; ++d) acc[d] = fmaf(pb, vs[j][d], acc[d]);
        }
      }
      m = m_new;
      first = false;
    }
  }
  if (!active) return;
  const float inv = 1.f / l;
  const size_t ob = base + (size_t)row * kD;
#pragma unroll
  for (int d = 0; d < kD; ++d) {
    const float ov = acc[d] * inv;
    o[ob + d] = from_f32<T>(ov);
    if (e.precise && o_prec) o_prec[ob + d] = ov;
  }
  float st;
  if (e.branch == BR_UNSHIFTED)
    st = e.inv_stat ? inv : inv_root(l, n);
  else if (e.branch == BR_SHIFTED)
    st = rho_exact(-m, r) * inv_root(l, n);
  else
    st = m + logf(l);
  stat[(size_t)bh * T_ + row] = st;
}

// Grid-stride over (row block, head) tiles; returns at once unless the
// resolved branch is one of branch_mask (the launch is then nearly free).
template <typename T>
__global__ void __launch_bounds__(kRows) attn_fwd_generic(algx_attn_config cfg, const T* __restrict__ q,
                                                          const T* __restrict__ k, const T* __restrict__ v,
                                                          const float* __restrict__ sink,
                                                          const float* __restrict__ guard, T* __restrict__ o,
                                                          float* __restrict__ o_prec, float* __restrict__ stat,
                                                          int H, int T_, int branch_mask, int BH) {
  // As the fast path's fallback this kernel may start before the fast kernel
  // ends (launch_dependent): wait for it, then let the next launch go.
  pdl_wait();
  pdl_trigger();
  const Eff e = resolve_variant(cfg, guard);
  if (!((branch_mask >> e.branch) & 1)) return;
  const int nblk = (T_ + kRows - 1) / kRows;
  for (int w = blockIdx.x; w < nblk * BH; w += gridDim.x) {
    attn_fwd_generic_tile<T>(cfg, q, k, v, sink, guard, o, o_prec, stat, H, T_, w % nblk, w / nblk, e);
    __syncthreads();
  }
}

// ------------------------------------------------------------------ backward
// di = sum_d dO*O (flash.py:633) per row, plus per-block partial sums of
// mass*di for the sink gradient (flash.py:694-705, 721-723).
template <typename T>
__global__ void __launch_bounds__(256) attn_di_kernel(algx_attn_config cfg, const float* __restrict__ guard,
                                                      const T* __restrict__ o, const float* __restrict__ o_prec,
                                                      const T* __restrict__ dout, const float* __restrict__ stat,
                                                      const float* __restrict__ sink, float* __restrict__ di,
                                                      float* __restrict__ sink_part, int H, int T_,
                                                      float* __restrict__ zero_acc, int* __restrict__ zero_tail) {
  pdl_wait();  // launched as a dependent: the forward's outputs are complete after this
  // no early launch_dependents (the backward's CTAs would wait on SMs this grid's later waves need)
  const Eff e = resolve_variant(cfg, guard);
  // The fast backward's fp32 dQ accumulator (zero_acc, rows of 64) and its
  // 256-byte counter area (zero_tail) are zeroed here, alongside the o / dO
  // reads, instead of by a separate memset (in both branches: under the range
  // guard the shifted branch's backward also runs on the tcgen05 path).
  if (zero_tail && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x < 64) zero_tail[threadIdx.x] = 0;
  const int bh = blockIdx.y, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kRows;
  const bool hs = cfg.has_sink != 0;
  float rb = 1.f, r;
  const float b = hs ? sink[h] : 0.f;
  if (hs && e.branch != BR_SOFTMAX) rb = rho_exact(e.clip ? fminf(b, cfg.clamp) : b, r);
  float part = 0.f;
  auto accumulate = [&](int row, float s) {
    di[(size_t)bh * T_ + row] = s;
    if (hs) {
      const float st = stat[(size_t)bh * T_ + row];
      float mass;
      if (e.branch == BR_SOFTMAX)
        mass = expf(b - st);
      else if (e.branch == BR_UNSHIFTED && e.inv_stat)
        mass = ipow(rb, cfg.n) * st;
      else
        mass = ipow(rb * st, cfg.n);
      part += mass * s;
    }
  };
  if (e.precise && o_prec) {
    // shifted guard fallback: the unrounded fp32 output, one warp per row
    for (int i = warp; i < kRows; i += 8) {
      const int row = row0 + i;
      if (row >= T_) break;
      const size_t off = ((size_t)bh * T_ + row) * kD + 2 * lane;
      float s = to_f32(dout[off]) * o_prec[off] + to_f32(dout[off + 1]) * o_prec[off + 1];
#pragma unroll
      for (int x = 16; x > 0; x >>= 1) s += __shfl_xor_sync(0xffffffffu, s, x);
      if (lane == 0) accumulate(row, s);
      // the tcgen05 backward of the shifted branch accumulates dQ here as well
      if (zero_acc) *reinterpret_cast<float2*>(zero_acc + off) = make_float2(0.f, 0.f);
    }
  } else {
    // 128-bit row loads, Vec<T>::TPR threads per row; all of a thread's rows
    // are loaded before any is used
    using V = Vec<T>;
    constexpr int kIt = kRows / (8 * V::RPW);
    const int sub = lane % V::TPR, rl = lane / V::TPR;
    uint4 ro[kIt], rd[kIt];
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int row = row0 + (warp + 8 * it) * V::RPW + rl;
      const bool ok = row < T_;
      const size_t off = ((size_t)bh * T_ + row) * kD + sub * V::N;
      ro[it] = ok ? ld_stream(o + off) : make_uint4(0, 0, 0, 0);
      rd[it] = ok ? ld_stream(dout + off) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int it = 0; it < kIt; ++it) {
      const int row = row0 + (warp + 8 * it) * V::RPW + rl;
      const bool ok = row < T_;
      float ov[V::N], dv[V::N];
      unpack<T>(ro[it], ov);
      unpack<T>(rd[it], dv);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) s = fmaf(dv[i], ov[i], s);
      s = row_sum<V::TPR>(s);
      if (ok && sub == 0) accumulate(row, s);
      if (zero_acc && ok) {
        float4* z = reinterpret_cast<float4*>(zero_acc + ((size_t)bh * T_ + row) * kD + sub * V::N);
#pragma unroll
        for (int c = 0; c < V::N / 4; ++c) z[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
#pragma unroll
  for (int x = 16; x > 0; x >>= 1) part += __shfl_xor_sync(0xffffffffu, part, x);
  if (!hs) return;
  __shared__ float red[8];
  if (lane == 0) red[warp] = part;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < 8; ++i) t += red[i];
    sink_part[(size_t)bh * gridDim.x + blockIdx.x] = t;
  }
}

// dsink[h] = -slope(h) * sum_{b, blocks} partial  (fixed summation order).
__global__ void attn_dsink_kernel(algx_attn_config cfg, const float* __restrict__ guard,
                                  const float* __restrict__ sink, const float* __restrict__ sink_part, int B,
                                  int H, int nblk, float* __restrict__ dsink) {
  const int h = threadIdx.x;
  if (h >= H) return;
  const Eff e = resolve_variant(cfg, guard);
  float s = 0.f;
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < nblk; ++i) s += sink_part[((size_t)b * H + h) * nblk + i];
  float slope = 1.f, r;
  if (e.branch != BR_SOFTMAX) {
    const float bb = e.clip ? fminf(sink[h], cfg.clamp) : sink[h];
    rho_exact(bb, r);
    slope = (float)cfg.n * r;
    if (e.clip && !(sink[h] < cfg.clamp)) slope = 0.f;
  }
  dsink[h] = -s * slope;
}

// p and ds of one score (flash.py:333-361), ds without the slope n.
struct PDs {
  float p, ds;
};
__device__ __forceinline__ PDs tile_grad(const Eff& e, const algx_attn_config& cfg, float s, float dp, float st,
                                         float dii) {
  float p, r = 1.f;
  if (e.branch == BR_SOFTMAX) {
    p = expf(s - st);
  } else {
    const float x = e.clip ? fminf(s, cfg.clamp) : s;
    const float rho = rho_sel(x, e.fast, r);
    p = (e.branch == BR_UNSHIFTED && e.inv_stat) ? ipow(rho, cfg.n) * st : ipow(rho * st, cfg.n);
  }
  float ds = p * (dp - dii);
  if (e.branch != BR_SOFTMAX) {
    ds *= r;
    if (e.clip && !(s < cfg.clamp)) ds = 0.f;
  }
  return {p, ds};
}

// dK, dV: one key row per thread; query tiles streamed through shared memory.
template <typename T>
__device__ __forceinline__ void attn_dkdv_generic_tile(algx_attn_config cfg, const T* __restrict__ q,
                                                           const T* __restrict__ k, const T* __restrict__ v,
                                                           const T* __restrict__ dout,
                                                           const float* __restrict__ stat,
                                                           const float* __restrict__ di,
                                                           const float* __restrict__ guard, T* __restrict__ dk,
                                                           T* __restrict__ dv, int T_, int blk_tile, int bh_tile, const Eff e) {
  extern __shared__ float smem[];
  float(*kown)[kD + 1] = reinterpret_cast<float(*)[kD + 1]>(smem);
  float(*vown)[kD + 1] = reinterpret_cast<float(*)[kD + 1]>(smem + kRows * (kD + 1));
  float(*qt)[kD] = reinterpret_cast<float(*)[kD]>(smem + 2 * kRows * (kD + 1));
  float(*dot)[kD] = reinterpret_cast<float(*)[kD]>(smem + 2 * kRows * (kD + 1) + kKT * kD);
  float* st = smem + 2 * kRows * (kD + 1) + 2 * kKT * kD;
  float* dit = st + kKT;
  const int bh = bh_tile;
  const int key0 = blk_tile * kRows;
  const int key = key0 + threadIdx.x;
  const bool active = key < T_;
  const size_t base = (size_t)bh * T_ * kD;
  for (int i = threadIdx.x; i < kRows * kD; i += kRows) {
    const int j = i / kD, d = i % kD, kk = key0 + j;
    kown[j][d] = kk < T_ ? to_f32(k[base + (size_t)kk * kD + d]) : 0.f;
    vown[j][d] = kk < T_ ? to_f32(v[base + (size_t)kk * kD + d]) : 0.f;
  }
  float dka[kD], dva[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) dka[d] = dva[d] = 0.f;
  const int t0 = key0 / kKT;
  const int ntiles = (T_ + kKT - 1) / kKT;
  for (int t = t0; t < ntiles; ++t) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKT * kD; i += kRows) {
      const int j = i / kD, d = i % kD, qi = t * kKT + j;
      qt[j][d] = qi < T_ ? to_f32(q[base + (size_t)qi * kD + d]) : 0.f;
      dot[j][d] = qi < T_ ? to_f32(dout[base + (size_t)qi * kD + d]) : 0.f;
    }
    if (threadIdx.x < kKT) {
      const int qi = t * kKT + threadIdx.x;
      st[threadIdx.x] = qi < T_ ? stat[(size_t)bh * T_ + qi] : 0.f;
      dit[threadIdx.x] = qi < T_ ? di[(size_t)bh * T_ + qi] : 0.f;
    }
    __syncthreads();
    if (!active) continue;
    for (int j = 0; j < kKT; ++j) {
      const int qi = t * kKT + j;
      if (qi < key || qi >= T_) continue;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < kD; ++d) {
        s = fmaf(qt[j][d], kown[threadIdx.x][d], s);
        dp = fmaf(dot[j][d], vown[threadIdx.x][d], dp);
      }
      const PDs g = tile_grad(e, cfg, s, dp, st[j], dit[j]);
      const float pb = round_io<T>(g.p), dsb = round_io<T>(g.ds);
#pragma unroll
      for (int d = 0; d < kD; ++d) {
        dva[d] = fmaf(pb, dot[j][d], dva[d]);
        dka[d] = fmaf(dsb, qt[j][d], dka[d]);
      }
    }
  }
  if (!active) return;
  const float slope = e.branch == BR_SOFTMAX ? 1.f : (float)cfg.n;
  const size_t ob = base + (size_t)key * kD;
#pragma unroll
  for (int d = 0; d < kD; ++d) {
    dk[ob + d] = from_f32<T>(dka[d] * slope);
    dv[ob + d] = from_f32<T>(dva[d]);
  }
}

// Grid-stride over (row block, head) tiles; returns at once unless the
// resolved branch is one of branch_mask (the launch is then nearly free).
template <typename T>
__global__ void __launch_bounds__(kRows) attn_dkdv_generic(algx_attn_config cfg, const T* __restrict__ q,
                                                           const T* __restrict__ k, const T* __restrict__ v,
                                                           const T* __restrict__ dout,
                                                           const float* __restrict__ stat,
                                                           const float* __restrict__ di,
                                                           const float* __restrict__ guard, T* __restrict__ dk,
                                                           T* __restrict__ dv, int T_, int branch_mask, int BH) {
  pdl_wait();  // see attn_fwd_generic
  pdl_trigger();
  const Eff e = resolve_variant(cfg, guard);
  if (!((branch_mask >> e.branch) & 1)) return;
  const int nblk = (T_ + kRows - 1) / kRows;
  for (int w = blockIdx.x; w < nblk * BH; w += gridDim.x) {
    attn_dkdv_generic_tile<T>(cfg, q, k, v, dout, stat, di, guard, dk, dv, T_, w % nblk, w / nblk, e);
    __syncthreads();
  }
}

// dQ: one query row per thread; key tiles streamed through shared memory.
template <typename T>
__device__ __forceinline__ void attn_dq_generic_tile(algx_attn_config cfg, const T* __restrict__ q,
                                                         const T* __restrict__ k, const T* __restrict__ v,
                                                         const T* __restrict__ dout, const float* __restrict__ stat,
                                                         const float* __restrict__ di,
                                                         const float* __restrict__ guard, T* __restrict__ dq,
                                                         int T_, int blk_tile, int bh_tile, const Eff e) {
  extern __shared__ float smem[];
  float(*qown)[kD + 1] = reinterpret_cast<float(*)[kD + 1]>(smem);
  float(*down)[kD + 1] = reinterpret_cast<float(*)[kD + 1]>(smem + kRows * (kD + 1));
  float(*kt)[kD] = reinterpret_cast<float(*)[kD]>(smem + 2 * kRows * (kD + 1));
  float(*vt)[kD] = reinterpret_cast<float(*)[kD]>(smem + 2 * kRows * (kD + 1) + kKT * kD);
  const int bh = bh_tile;
  const int row0 = blk_tile * kRows;
  const int row = row0 + threadIdx.x;
  const bool active = row < T_;
  const size_t base = (size_t)bh * T_ * kD;
  for (int i = threadIdx.x; i < kRows * kD; i += kRows) {
    const int j = i / kD, d = i % kD, qi = row0 + j;
    qown[j][d] = qi < T_ ? to_f32(q[base + (size_t)qi * kD + d]) : 0.f;
    down[j][d] = qi < T_ ? to_f32(dout[base + (size_t)qi * kD + d]) : 0.f;
  }
  const float myst = active ? stat[(size_t)bh * T_ + row] : 0.f;
  const float mydi = active ? di[(size_t)bh * T_ + row] : 0.f;
  float dqa[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) dqa[d] = 0.f;
  const int last = min(T_, row0 + kRows) - 1;
  const int ntiles = last / kKT + 1;
  for (int t = 0; t < ntiles; ++t) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKT * kD; i += kRows) {
      const int j = i / kD, d = i % kD, kk = t * kKT + j;
      kt[j][d] = kk < T_ ? to_f32(k[base + (size_t)kk * kD + d]) : 0.f;
      vt[j][d] = kk < T_ ? to_f32(v[base + (size_t)kk * kD + d]) : 0.f;
    }
    __syncthreads();
    if (!active) continue;
    for (int j = 0; j < kKT; ++j) {
      const int kk = t * kKT + j;
      if (kk > row) break;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < kD; ++d) {
        s = fmaf(qown[threadIdx.x][d], kt[j][d], s);
        dp = fmaf(down[threadIdx.x][d], vt[j][d], dp);
      }
      const PDs g = tile_grad(e, cfg, s, dp, myst, mydi);
      const float dsb = round_io<T>(g.ds);
#pragma unroll
      for (int d = 0; d < kD; ++d) dqa[d] = fmaf(dsb, kt[j][d], dqa[d]);
    }
  }
  if (!active) return;
  const float f = (e.branch == BR_SOFTMAX ? 1.f : (float)cfg.n) * cfg.scale;
  const size_t ob = base + (size_t)row * kD;
#pragma unroll
  for (int d = 0; d < kD; ++d) dq[ob + d] = from_f32<T>(dqa[d] * f);
}

// Grid-stride over (row block, head) tiles; returns at once unless the
// resolved branch is one of branch_mask (the launch is then nearly free).
template <typename T>
__global__ void __launch_bounds__(kRows) attn_dq_generic(algx_attn_config cfg, const T* __restrict__ q,
                                                         const T* __restrict__ k, const T* __restrict__ v,
                                                         const T* __restrict__ dout, const float* __restrict__ stat,
                                                         const float* __restrict__ di,
                                                         const float* __restrict__ guard, T* __restrict__ dq,
                                                         int T_, int branch_mask, int BH) {
  pdl_wait();  // see attn_fwd_generic
  pdl_trigger();
  const Eff e = resolve_variant(cfg, guard);
  if (!((branch_mask >> e.branch) & 1)) return;
  const int nblk = (T_ + kRows - 1) / kRows;
  for (int w = blockIdx.x; w < nblk * BH; w += gridDim.x) {
    attn_dq_generic_tile<T>(cfg, q, k, v, dout, stat, di, guard, dq, T_, w % nblk, w / nblk, e);
    __syncthreads();
  }
}

constexpr size_t kGenericBwdSmem = (2 * kRows * (kD + 1) + 2 * kKT * kD + 2 * kKT) * sizeof(float);

int check_attn(const algx_attn_config* cfg, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype) {
  ALGX_REQUIRE(cfg, "attention: NULL config");
  ALGX_REQUIRE(D == kD, "attention: head dim must be 64");
  ALGX_REQUIRE(B >= 1 && H >= 1 && T >= 1, "attention: empty shape");
  ALGX_REQUIRE(T <= (1 << 23) && B * H <= 65535, "attention: shape too large");
  ALGX_REQUIRE(H <= 1024, "attention: at most 1024 heads");
  ALGX_REQUIRE(dtype == ALGX_F32 || dtype == ALGX_BF16, "attention: dtype must be float32 or bfloat16");
  ALGX_REQUIRE(cfg->kind == ALGX_ATTN_ASINH || cfg->kind == ALGX_ATTN_SOFTMAX, "attention: unknown kind");
  if (cfg->kind == ALGX_ATTN_ASINH) {
    ALGX_REQUIRE(cfg->n >= 2 && (cfg->n & (cfg->n - 1)) == 0, "asinh kernel needs n to be a power of two");
    ALGX_REQUIRE(cfg->mode >= ALGX_MODE_CLIPPED && cfg->mode <= ALGX_MODE_GUARDED, "attention: unknown mode");
  }
  return ALGX_OK;
}

// ------------------------------------------------------------------ fused QK-norm backward
// Backward of the QK RMS norm (kernels/qk_norm.py:45-56) applied to the
// attention's dq and dk, in place: dq_x holds dq (bf16 from the generic
// kernels) or, when the fast path ran the backward (tc_bwd_covers), dq is
// read from the fp32 accumulator as bf16(acc * n * scale), the rounding of
// dq_finish_kernel; dk_x holds dk. Per row the arithmetic is that of
// qknorm_bwd_kernel, so dx is bit-identical to the composed calls. dgain:
// per-CTA column partials, then the last CTA to finish sums them in a fixed
// order (deterministic for a given grid) and resets the arrival counter.
constexpr int kEpiThreads = 512;
constexpr int kEpiUnroll = 4;

// All loads of a thread's kEpiUnroll rows are issued before any is used, so
// that enough bytes are in flight to keep HBM busy at one CTA per SM.
// x and dx_out are head-major (tok_stride 0) or blocks of a token-major
// (B, T, 3, H, D) tensor (tok_stride 3H); dy_in (when not FROM_ACC) and acc
// are head-major. dy_in may equal dx_out (the in-place head-major call).
template <typename T, bool FROM_ACC, bool PACKED>
__device__ __forceinline__ void qk_rows_bwd(const T* __restrict__ x, const float* __restrict__ gain, const T* dy_in,
                                            T* dx_out, const float* __restrict__ acc, float f,
                                            const float* __restrict__ rot_cos, const float* __restrict__ rot_sin,
                                            int T_, int H, int tok_stride, int64_t rows, float eps,
                                            float (&part)[Vec<T>::N]) {
  using V = Vec<T>;
  constexpr int kA = FROM_ACC ? V::N / 4 : 1;  // 16-byte chunks of fp32 accumulator per thread and row
  const int lane = threadIdx.x & 31, sub = lane % V::TPR, rl = lane / V::TPR;
  float g[V::N];
#pragma unroll
  for (int i = 0; i < V::N; ++i) g[i] = gain[sub * V::N + i];
  const int64_t warps = (int64_t)gridDim.x * (kEpiThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kEpiThreads / 32) + (threadIdx.x >> 5);
  for (int64_t r0 = w * V::RPW * kEpiUnroll; r0 < rows; r0 += warps * V::RPW * kEpiUnroll) {
    uint4 rx[kEpiUnroll], rd[kEpiUnroll][kA];
#pragma unroll
    for (int u = 0; u < kEpiUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      const bool ok = row < rows;
      const int64_t xrow = PACKED ? tok_row(row, T_, H, tok_stride) : row;
      rx[u] = ok ? ld_stream(x + xrow * kD + sub * V::N) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c = 0; c < kA; ++c) {
        if constexpr (FROM_ACC)
          rd[u][c] = ok ? ld_stream(acc + row * kD + sub * V::N + 4 * c) : make_uint4(0, 0, 0, 0);
        else
          rd[u][c] = ok ? *reinterpret_cast<const uint4*>(dy_in + row * kD + sub * V::N) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kEpiUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      float xv[V::N], dv[V::N];
      unpack<T>(rx[u], xv);
      if constexpr (FROM_ACC) {
#pragma unroll
        for (int c = 0; c < kA; ++c) {
          dv[4 * c + 0] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rd[u][c].x) * f));
          dv[4 * c + 1] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rd[u][c].y) * f));
          dv[4 * c + 2] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rd[u][c].z) * f));
          dv[4 * c + 3] = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rd[u][c].w) * f));
        }
      } else {
        unpack<T>(rd[u][0], dv);
      }
      if (rot_cos) rotate_half<T, true>(dv, rot_cos, rot_sin, row % T_, sub);
      float ss = 0.f, sdg = 0.f;
#pragma unroll
      for (int i = 0; i < V::N; ++i) {
        ss = fmaf(xv[i], xv[i], ss);
        sdg = fmaf(dv[i] * g[i], xv[i], sdg);
      }
      ss = row_sum<V::TPR>(ss);
      sdg = row_sum<V::TPR>(sdg);
      const float tau = rsqrtf(ss * (1.0f / kD) + eps);
      const float corr = tau * tau * tau * sdg * (1.0f / kD);
      float out[V::N];
#pragma unroll
      for (int i = 0; i < V::N; ++i) {
        out[i] = (dv[i] * g[i]) * tau - xv[i] * corr;
        part[i] = fmaf(dv[i], xv[i] * tau, part[i]);
      }
      const int64_t orow = PACKED ? tok_row(row, T_, H, tok_stride) : row;
      if (row < rows) *reinterpret_cast<uint4*>(dx_out + orow * kD + sub * V::N) = pack<T>(out);
    }
  }
}

// dv_out (token-major block, tok_stride) = dv_in (head-major), row by row.
template <typename T>
__device__ __forceinline__ void copy_rows_to_tokens(const T* __restrict__ dv_in, T* __restrict__ dv_out, int T_, int H,
                                                    int tok_stride, int64_t rows) {
  using V = Vec<T>;
  const int lane = threadIdx.x & 31, sub = lane % V::TPR, rl = lane / V::TPR;
  const int64_t warps = (int64_t)gridDim.x * (kEpiThreads / 32);
  const int64_t w = (int64_t)blockIdx.x * (kEpiThreads / 32) + (threadIdx.x >> 5);
  for (int64_t r0 = w * V::RPW * kEpiUnroll; r0 < rows; r0 += warps * V::RPW * kEpiUnroll) {
    uint4 raw[kEpiUnroll];
#pragma unroll
    for (int u = 0; u < kEpiUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      raw[u] = row < rows ? ld_stream(dv_in + row * kD + sub * V::N) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kEpiUnroll; ++u) {
      const int64_t row = r0 + u * V::RPW + rl;
      if (row < rows) *reinterpret_cast<uint4*>(dv_out + tok_row(row, T_, H, tok_stride) * kD + sub * V::N) = raw[u];
    }
  }
}

template <typename T, bool PACKED>
__global__ void __launch_bounds__(kEpiThreads) qknorm_attn_bwd_kernel(
    algx_attn_config cfg, const float* __restrict__ guard, int fast, const float* __restrict__ dq_acc,
    const T* __restrict__ q, const float* __restrict__ gain_q, const T* __restrict__ k,
    const float* __restrict__ gain_k, const float* __restrict__ rot_cos, const float* __restrict__ rot_sin, int T_,
    T* dq_x, T* dk_x, float* __restrict__ partial, unsigned* counter, float* __restrict__ dgain_q,
    float* __restrict__ dgain_k, int64_t rows, float eps, int H, int tok_stride, const T* dq_in, const T* dk_in,
    const T* __restrict__ dv_in, T* __restrict__ dv_out) {
  pdl_wait();  // launched as a dependent of the attention backward
  using V = Vec<T>;
  __shared__ float red[kEpiThreads / 32 * V::RPW][2 * kD];  // per row slot of a warp: q and k column sums
  __shared__ float fin[kEpiThreads / (2 * kD)][2 * kD];
  __shared__ bool last;
  const bool use_acc = fast && tc_bwd_covers(cfg, resolve_variant(cfg, guard));
  float pq[V::N], pk[V::N];
#pragma unroll
  for (int i = 0; i < V::N; ++i) pq[i] = pk[i] = 0.f;
  if (use_acc)
    qk_rows_bwd<T, true, PACKED>(q, gain_q, nullptr, dq_x, dq_acc, (float)cfg.n * cfg.scale, rot_cos, rot_sin, T_,
                                 H, tok_stride, rows, eps, pq);
  else
    qk_rows_bwd<T, false, PACKED>(q, gain_q, dq_in, dq_x, nullptr, 1.f, rot_cos, rot_sin, T_, H, tok_stride, rows,
                                  eps, pq);
  qk_rows_bwd<T, false, PACKED>(k, gain_k, dk_in, dk_x, nullptr, 1.f, rot_cos, rot_sin, T_, H, tok_stride, rows, eps,
                                pk);
  if constexpr (PACKED) copy_rows_to_tokens<T>(dv_in, dv_out, T_, H, tok_stride, rows);
  // CTA column sums: slot (warp, row-in-warp) holds its threads' columns
  const int lane = threadIdx.x & 31, sub = lane % V::TPR, rl = lane / V::TPR;
  const int slot = (threadIdx.x >> 5) * V::RPW + rl;
#pragma unroll
  for (int i = 0; i < V::N; ++i) {
    red[slot][sub * V::N + i] = pq[i];
    red[slot][kD + sub * V::N + i] = pk[i];
  }
  __syncthreads();
  if (threadIdx.x < 2 * kD) {
    float sum = 0.f;
    for (int r = 0; r < kEpiThreads / 32 * V::RPW; ++r) sum += red[r][threadIdx.x];
    partial[(int64_t)blockIdx.x * 2 * kD + threadIdx.x] = sum;
    __threadfence();
  }
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int c = threadIdx.x % (2 * kD), part = threadIdx.x / (2 * kD);
  constexpr int kParts = kEpiThreads / (2 * kD);
  float sum = 0.f;
#pragma unroll 8
  for (int b = part; b < (int)gridDim.x; b += kParts) sum += __ldcg(partial + (int64_t)b * 2 * kD + c);
  fin[part][c] = sum;
  __syncthreads();
  if (threadIdx.x < 2 * kD) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kParts; ++i) t += fin[i][threadIdx.x];
    if (threadIdx.x < kD)
      dgain_q[threadIdx.x] = t;
    else
      dgain_k[threadIdx.x - kD] = t;
  }
  if (threadIdx.x == 0) *counter = 0u;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Grid of the generic kernels: every (row block, head) tile when they do the
// work; when the fast kernels ran they only stand by for the shifted
// fallback, and a grid of four CTAs per SM returns almost at once.
unsigned generic_grid(int64_t BH, int64_t T, bool fast) {
  const int64_t tiles = BH * ((T + kRows - 1) / kRows);
  return (unsigned)(fast ? std::min<int64_t>(tiles, 148 * 4) : tiles);
}

}  // namespace

// Backward workspace layout: [di (B*H*T fp32) | sink partials | fast-path area].
size_t ws_off_sink(int64_t B, int64_t H, int64_t T) { return align256((size_t)B * H * T * sizeof(float)); }
size_t ws_off_tc(int64_t B, int64_t H, int64_t T) {
  const int64_t nblk = (T + kRows - 1) / kRows;
  return ws_off_sink(B, H, T) + align256((size_t)B * H * nblk * sizeof(float));
}
// The fused QK-norm backward appends its dgain partials and, for calls where
// the fast path does not zero its spare bytes, its own arrival counter.
constexpr int kEpiBlocks = 148;
size_t ws_off_epi(int64_t B, int64_t H, int64_t T, int64_t D) {
  return align256(ws_off_tc(B, H, T) + tc_attn_bwd_workspace(B, H, T, D));
}
size_t epi_bytes() { return align256((size_t)kEpiBlocks * 2 * kD * sizeof(float)) + 256; }

}  // namespace algx

using namespace algx;

extern "C" {

int algx_attn_prepare(const algx_attn_config* cfg, const void* q, const void* k, const void* v, const float* sink,
                      void* q_scaled, float* guard, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                      void* stream) {
  if (int s = check_attn(cfg, B, H, T, D, dtype)) return s;
  ALGX_REQUIRE(q && k && v && q_scaled && guard, "attn_prepare: NULL pointer");
  ALGX_REQUIRE(!cfg->has_sink || sink, "attn_prepare: has_sink without a sink pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ALGX_CUDA(cudaMemsetAsync(guard, 0, 4 * sizeof(float), st));
  const int64_t rows = B * H * T;
  const int64_t rows_per_block = (kPrepThreads / 32) * (dtype == ALGX_BF16 ? 4 : 2);
  const int gx = (int)std::min<int64_t>((rows + rows_per_block - 1) / rows_per_block, 148 * 8);
  dim3 grid(gx, 3);
  const float* sk = cfg->has_sink ? sink : nullptr;
  if (dtype == ALGX_BF16)
    attn_prepare_kernel<__nv_bfloat16><<<grid, kPrepThreads, 0, st>>>(
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, sk, (int)H,
        (__nv_bfloat16*)q_scaled, guard, rows, cfg->scale);
  else
    attn_prepare_kernel<float><<<grid, kPrepThreads, 0, st>>>((const float*)q, (const float*)k, (const float*)v,
                                                              sk, (int)H, (float*)q_scaled, guard, rows,
                                                              cfg->scale);
  ALGX_LAUNCHED("attn_prepare launch");
  return ALGX_OK;
}

}  // extern "C"

namespace algx {
namespace {
// Shared body of the head-major and packed prologues: q, k, v point at the
// first row of each block, in_stride as in qknorm_attn_prepare_kernel.
int qknorm_prepare_impl(const algx_attn_config* cfg, const void* q, const void* k, const void* v,
                        const float* gain_q, const float* gain_k, const float* rope_cos, const float* rope_sin,
                        int64_t rope_rows, const float* sink, void* q_scaled, void* k_norm, void* v_heads,
                        float* guard, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype, float eps,
                        int in_stride, void* stream) {
  if (int s = check_attn(cfg, B, H, T, D, dtype)) return s;
  ALGX_REQUIRE(q && k && v && gain_q && gain_k && q_scaled && k_norm && guard, "qknorm_attn_prepare: NULL pointer");
  ALGX_REQUIRE((rope_cos == nullptr) == (rope_sin == nullptr), "qknorm_attn_prepare: give both rotary tables or none");
  ALGX_REQUIRE(!rope_cos || rope_rows >= T, "qknorm_attn_prepare: rotary tables need at least T rows");
  ALGX_REQUIRE(!cfg->has_sink || sink, "qknorm_attn_prepare: has_sink without a sink pointer");
  ALGX_REQUIRE(eps > 0.f, "qknorm_attn_prepare: eps must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ALGX_CUDA(cudaMemsetAsync(guard, 0, 4 * sizeof(float), st));
  const int64_t rows = B * H * T;
  const int64_t rows_per_block = (kPrepThreads / 32) * (dtype == ALGX_BF16 ? 4 : 2) * 4;
  const int gx = (int)std::min<int64_t>((rows + rows_per_block - 1) / rows_per_block, 148 * 8);
  dim3 grid(gx, 3);
  const float* sk = cfg->has_sink ? sink : nullptr;
  auto launch = [&](auto kern, auto tag) {
    using TT = decltype(tag);
    kern<<<grid, kPrepThreads, 0, st>>>((const TT*)q, (const TT*)k, (const TT*)v, gain_q, gain_k, rope_cos, rope_sin,
                                        sk, (int)H, (int)T, (TT*)q_scaled, (TT*)k_norm, guard, rows, cfg->scale, eps,
                                        in_stride, (TT*)v_heads);
  };
  ALGX_REQUIRE(in_stride == 0 || v_heads, "qknorm_attn_prepare: the packed layout needs v_heads");
  const bool packed = in_stride != 0;
  if (dtype == ALGX_BF16) {
    if (packed)
      rope_cos ? launch(qknorm_attn_prepare_kernel<__nv_bfloat16, true, true>, __nv_bfloat16{})
               : launch(qknorm_attn_prepare_kernel<__nv_bfloat16, false, true>, __nv_bfloat16{});
    else
      rope_cos ? launch(qknorm_attn_prepare_kernel<__nv_bfloat16, true, false>, __nv_bfloat16{})
               : launch(qknorm_attn_prepare_kernel<__nv_bfloat16, false, false>, __nv_bfloat16{});
  } else {
    if (packed)
      rope_cos ? launch(qknorm_attn_prepare_kernel<float, true, true>, float{})
               : launch(qknorm_attn_prepare_kernel<float, false, true>, float{});
    else
      rope_cos ? launch(qknorm_attn_prepare_kernel<float, true, false>, float{})
               : launch(qknorm_attn_prepare_kernel<float, false, false>, float{});
  }
  ALGX_LAUNCHED("qknorm_attn_prepare launch");
  return ALGX_OK;
}
}  // namespace
}  // namespace algx

extern "C" {

int algx_qknorm_attn_prepare(const algx_attn_config* cfg, const void* q, const void* k, const void* v,
                             const float* gain_q, const float* gain_k, const float* rope_cos, const float* rope_sin,
                             int64_t rope_rows, const float* sink, void* q_scaled, void* k_norm, float* guard,
                             int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype, float eps, void* stream) {
  return qknorm_prepare_impl(cfg, q, k, v, gain_q, gain_k, rope_cos, rope_sin, rope_rows, sink, q_scaled, k_norm,
                             nullptr, guard, B, H, T, D, dtype, eps, 0, stream);
}

int algx_qknorm_attn_prepare_packed(const algx_attn_config* cfg, const void* qkv, const float* gain_q,
                                    const float* gain_k, const float* rope_cos, const float* rope_sin,
                                    int64_t rope_rows, const float* sink, void* q_scaled, void* k_norm, void* v_heads,
                                    float* guard, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                                    float eps, void* stream) {
  ALGX_REQUIRE(qkv && v_heads, "qknorm_attn_prepare_packed: NULL pointer");
  ALGX_REQUIRE(H > 0 && 3 * H <= INT32_MAX, "qknorm_attn_prepare_packed: bad head count");
  ALGX_REQUIRE(B >= 0 && T > 0 && B * H * T <= INT32_MAX, "qknorm_attn_prepare_packed: B*H*T must be below 2^31");
  const size_t es = dtype == ALGX_BF16 ? 2 : 4;
  const char* base = static_cast<const char*>(qkv);
  const size_t blk = (size_t)H * (size_t)D * es;  // bytes between the q, k and v blocks of a token row
  return qknorm_prepare_impl(cfg, base, base + blk, base + 2 * blk, gain_q, gain_k, rope_cos, rope_sin, rope_rows,
                             sink, q_scaled, k_norm, v_heads, guard, B, H, T, D, dtype, eps, (int)(3 * H), stream);
}

int algx_attn_fwd(const algx_attn_config* cfg, const void* q_scaled, const void* k, const void* v, const float* sink,
                  const float* guard, void* o, float* o_precise, float* stat, int64_t B, int64_t H, int64_t T,
                  int64_t D, int32_t dtype, void* stream) {
  if (int s = check_attn(cfg, B, H, T, D, dtype)) return s;
  ALGX_REQUIRE(q_scaled && k && v && guard && o && stat, "attn_fwd: NULL pointer");
  ALGX_REQUIRE(!cfg->has_sink || sink, "attn_fwd: has_sink without a sink pointer");
  ALGX_REQUIRE(cfg->kind != ALGX_ATTN_ASINH || cfg->mode != ALGX_MODE_GUARDED || o_precise,
               "attn_fwd: guarded mode needs o_precise");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int mask = 7;
  bool fast = false;
  if (int s = tc_attn_fwd(*cfg, q_scaled, k, v, sink, guard, o, o_precise, stat, B, H, T, dtype, st, &fast))
    return s;
  if (fast) {
    // The fast kernel covers the unshifted branch, which the clipped link
    // always takes, and under the range guard the shifted branch as well.
    if (cfg->mode == ALGX_MODE_CLIPPED || cfg->mode == ALGX_MODE_GUARDED) return ALGX_OK;
    mask = 1 << BR_SHIFTED | 1 << BR_SOFTMAX;
  }
  const unsigned grid = generic_grid(B * H, T, fast);
  if (fast)  // only the fast path's bf16 fallback: overlaps the fast kernel's tail
    ALGX_CUDA(launch_dependent(attn_fwd_generic<__nv_bfloat16>, grid, kRows, 0, st, *cfg,
                               (const __nv_bfloat16*)q_scaled, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                               sink, guard, (__nv_bfloat16*)o, o_precise, stat, (int)H, (int)T, mask, (int)(B * H)));
  else if (dtype == ALGX_BF16)
    attn_fwd_generic<__nv_bfloat16><<<grid, kRows, 0, st>>>(*cfg, (const __nv_bfloat16*)q_scaled,
                                                             (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                                                             sink, guard, (__nv_bfloat16*)o, o_precise, stat,
                                                             (int)H, (int)T, mask, (int)(B * H));
  else
    attn_fwd_generic<float><<<grid, kRows, 0, st>>>(*cfg, (const float*)q_scaled, (const float*)k, (const float*)v,
                                                    sink, guard, (float*)o, o_precise, stat, (int)H, (int)T, mask,
                                                    (int)(B * H));
  ALGX_LAUNCHED("attn_fwd_generic launch");
  return ALGX_OK;
}

size_t algx_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D) {
  return ws_off_tc(B, H, T) + tc_attn_bwd_workspace(B, H, T, D);
}

// The attention backward launch group. With finish_dq false and the fast
// path taken (*fast), the fp32 accumulator holds dq unscaled whenever
// tc_bwd_covers(cfg, branch); otherwise dq holds the generic kernels' result.
static int attn_bwd_core(const algx_attn_config* cfg, const void* q_scaled, const void* k, const void* v,
                         const float* sink, const float* guard, const void* o, const float* o_precise,
                         const float* stat, const void* dout, void* dq, void* dk, void* dv, float* dsink, int64_t B,
                         int64_t H, int64_t T, int32_t dtype, void* workspace, cudaStream_t st, bool finish_dq,
                         bool* fast_out) {
  char* ws = static_cast<char*>(workspace);
  float* di = reinterpret_cast<float*>(ws);
  float* sink_part = reinterpret_cast<float*>(ws + ws_off_sink(B, H, T));
  void* tc_ws = ws + ws_off_tc(B, H, T);
  const int nblk = (int)((T + kRows - 1) / kRows);
  dim3 grid((unsigned)nblk, (unsigned)(B * H));
  // when the fast backward will run, the di pass zeroes its accumulator too
  const bool fast_next = tc_attn_bwd_eligible(*cfg, T, dtype);
  float* zero_acc = fast_next ? static_cast<float*>(tc_ws) : nullptr;
  int* zero_tail =  // the 256 bytes after the accumulator
      fast_next ? reinterpret_cast<int*>(static_cast<char*>(tc_ws) + tc_attn_bwd_workspace(B, H, T, kD) - 256) : nullptr;
  if (dtype == ALGX_BF16)
    ALGX_CUDA(launch_dependent(attn_di_kernel<__nv_bfloat16>, grid, 256, 0, st, *cfg, guard,
                               (const __nv_bfloat16*)o, o_precise, (const __nv_bfloat16*)dout, stat, sink, di,
                               sink_part, (int)H, (int)T, zero_acc, zero_tail));
  else
    ALGX_CUDA(launch_dependent(attn_di_kernel<float>, grid, 256, 0, st, *cfg, guard, (const float*)o, o_precise,
                               (const float*)dout, stat, sink, di, sink_part, (int)H, (int)T, zero_acc,
                               zero_tail));
  ALGX_LAUNCHED("attn_di launch");
  if (cfg->has_sink) {
    attn_dsink_kernel<<<1, (unsigned)((H + 31) / 32 * 32), 0, st>>>(*cfg, guard, sink, sink_part, (int)B, (int)H,
                                                                    nblk, dsink);
    ALGX_LAUNCHED("attn_dsink launch");
  }
  int mask = 7;
  bool fast = false;
  if (int s = tc_attn_bwd(*cfg, q_scaled, k, v, dout, stat, di, guard, dq, dk, dv, tc_ws, B, H, T, dtype, st,
                          finish_dq, fast_next, &fast))
    return s;
  *fast_out = fast;
  if (fast) {
    // the tcgen05 kernels cover the clipped link, and under the range guard
    // both branches (tc_bwd_covers): no CUDA-core stand-by is needed
    if (cfg->mode == ALGX_MODE_CLIPPED || cfg->mode == ALGX_MODE_GUARDED) return ALGX_OK;
    mask = 1 << BR_SHIFTED | 1 << BR_SOFTMAX;
  }
  const unsigned ggrid = generic_grid(B * H, T, fast);
  int dev = 0;
  ALGX_CUDA(cudaGetDevice(&dev));
  static bool attr_set[64][2] = {};
  if (dev >= 0 && dev < 64 && !attr_set[dev][dtype]) {
    if (dtype == ALGX_BF16) {
      ALGX_CUDA(cudaFuncSetAttribute(attn_dkdv_generic<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kGenericBwdSmem));
      ALGX_CUDA(cudaFuncSetAttribute(attn_dq_generic<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kGenericBwdSmem));
    } else {
      ALGX_CUDA(cudaFuncSetAttribute(attn_dkdv_generic<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kGenericBwdSmem));
      ALGX_CUDA(cudaFuncSetAttribute(attn_dq_generic<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kGenericBwdSmem));
    }
    attr_set[dev][dtype] = true;
  }
  const int bh = (int)(B * H);
  if (fast) {  // only the fast path's bf16 fallback: overlaps the fast kernel's tail
    ALGX_CUDA(launch_dependent(attn_dkdv_generic<__nv_bfloat16>, ggrid, kRows, kGenericBwdSmem, st, *cfg,
                               (const __nv_bfloat16*)q_scaled, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                               (const __nv_bfloat16*)dout, stat, di, guard, (__nv_bfloat16*)dk, (__nv_bfloat16*)dv,
                               (int)T, mask, bh));
    ALGX_CUDA(launch_dependent(attn_dq_generic<__nv_bfloat16>, ggrid, kRows, kGenericBwdSmem, st, *cfg,
                               (const __nv_bfloat16*)q_scaled, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
                               (const __nv_bfloat16*)dout, stat, di, guard, (__nv_bfloat16*)dq, (int)T, mask, bh));
  } else if (dtype == ALGX_BF16) {
    attn_dkdv_generic<__nv_bfloat16><<<ggrid, kRows, kGenericBwdSmem, st>>>(
        *cfg, (const __nv_bfloat16*)q_scaled, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
        (const __nv_bfloat16*)dout, stat, di, guard, (__nv_bfloat16*)dk, (__nv_bfloat16*)dv, (int)T, mask, bh);
    attn_dq_generic<__nv_bfloat16><<<ggrid, kRows, kGenericBwdSmem, st>>>(
        *cfg, (const __nv_bfloat16*)q_scaled, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v,
        (const __nv_bfloat16*)dout, stat, di, guard, (__nv_bfloat16*)dq, (int)T, mask, bh);
  } else {
    attn_dkdv_generic<float><<<ggrid, kRows, kGenericBwdSmem, st>>>(*cfg, (const float*)q_scaled, (const float*)k,
                                                                    (const float*)v, (const float*)dout, stat, di,
                                                                    guard, (float*)dk, (float*)dv, (int)T, mask, bh);
    attn_dq_generic<float><<<ggrid, kRows, kGenericBwdSmem, st>>>(*cfg, (const float*)q_scaled, (const float*)k,
                                                                  (const float*)v, (const float*)dout, stat, di,
                                                                  guard, (float*)dq, (int)T, mask, bh);
  }
  count_launches(1);  // two kernels above, one counted by the macro
  ALGX_LAUNCHED("attn_bwd_generic launch");
  return ALGX_OK;
}

int algx_attn_bwd(const algx_attn_config* cfg, const void* q_scaled, const void* k, const void* v, const float* sink,
                  const float* guard, const void* o, const float* o_precise, const float* stat, const void* dout,
                  void* dq, void* dk, void* dv, float* dsink, int64_t B, int64_t H, int64_t T, int64_t D,
                  int32_t dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (int s = check_attn(cfg, B, H, T, D, dtype)) return s;
  ALGX_REQUIRE(q_scaled && k && v && guard && o && stat && dout && dq && dk && dv, "attn_bwd: NULL pointer");
  ALGX_REQUIRE(!cfg->has_sink || (sink && dsink), "attn_bwd: has_sink needs sink and dsink");
  ALGX_REQUIRE(workspace && workspace_bytes >= algx_attn_bwd_workspace_size(B, H, T, D),
               "attn_bwd: workspace too small (see algx_attn_bwd_workspace_size)");
  bool fast = false;
  return attn_bwd_core(cfg, q_scaled, k, v, sink, guard, o, o_precise, stat, dout, dq, dk, dv, dsink, B, H, T, dtype,
                       workspace, static_cast<cudaStream_t>(stream), true, &fast);
}

size_t algx_qknorm_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D) {
  return ws_off_epi(B, H, T, D) + epi_bytes();
}

}  // extern "C"

namespace algx {
namespace {
// Shared body of the head-major and packed backward calls. q_src/k_src: the
// raw (pre-norm) q and k, head-major (tok_stride 0) or blocks of the packed
// (B, T, 3, H, D) input (tok_stride 3H); dq_out/dk_out likewise. The
// attention backward writes its dq, dk, dv into dq_h, dk_h, dv_h (head-major);
// with dv_out set, the epilogue also copies dv_h into it.
int qknorm_attn_bwd_impl(const algx_attn_config* cfg, const void* q_src, const void* k_src, const float* gain_q,
                         const float* gain_k, const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                         const void* q_scaled, const void* k_norm, const void* v, const float* sink,
                         const float* guard, const void* o, const float* o_precise, const float* stat,
                         const void* dout, void* dq_h, void* dk_h, void* dv_h, void* dq_out, void* dk_out,
                         void* dv_out, int tok_stride, float* dgain_q, float* dgain_k, float* dsink, int64_t B,
                         int64_t H, int64_t T, int64_t D, int32_t dtype, float eps, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (int s = check_attn(cfg, B, H, T, D, dtype)) return s;
  ALGX_REQUIRE(q_src && k_src && gain_q && gain_k && q_scaled && k_norm && v && guard && o && stat && dout && dq_h &&
                   dk_h && dv_h && dq_out && dk_out && dgain_q && dgain_k,
               "qknorm_attn_bwd: NULL pointer");
  ALGX_REQUIRE(!cfg->has_sink || (sink && dsink), "qknorm_attn_bwd: has_sink needs sink and dsink");
  ALGX_REQUIRE(eps > 0.f, "qknorm_attn_bwd: epsilon must be positive");
  ALGX_REQUIRE((rope_cos == nullptr) == (rope_sin == nullptr), "qknorm_attn_bwd: give both rotary tables or none");
  ALGX_REQUIRE(!rope_cos || rope_rows >= T, "qknorm_attn_bwd: rotary tables need at least T rows");
  ALGX_REQUIRE(workspace && workspace_bytes >= algx_qknorm_attn_bwd_workspace_size(B, H, T, D),
               "qknorm_attn_bwd: workspace too small (see algx_qknorm_attn_bwd_workspace_size)");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bool fast = false;
  if (int s = attn_bwd_core(cfg, q_scaled, k_norm, v, sink, guard, o, o_precise, stat, dout, dq_h, dk_h, dv_h, dsink,
                            B, H, T, dtype, workspace, st, false, &fast))
    return s;
  char* ws = static_cast<char*>(workspace);
  const float* acc = reinterpret_cast<const float*>(ws + ws_off_tc(B, H, T));
  float* partial = reinterpret_cast<float*>(ws + ws_off_epi(B, H, T, D));
  unsigned* counter;
  if (fast) {  // zeroed with the accumulator
    counter = reinterpret_cast<unsigned*>(ws + ws_off_tc(B, H, T) + tc_attn_bwd_spare_offset(B, H, T, D));
  } else {
    counter = reinterpret_cast<unsigned*>(ws + ws_off_epi(B, H, T, D) + epi_bytes() - 256);
    ALGX_CUDA(cudaMemsetAsync(counter, 0, sizeof(unsigned), st));
  }
  const int64_t rows = B * H * T;
  auto launch = [&](auto tag, auto packed) {
    using TT = decltype(tag);
    return launch_dependent(qknorm_attn_bwd_kernel<TT, decltype(packed)::value>, kEpiBlocks, kEpiThreads, 0, st,
                            *cfg, guard,
                            (dtype == ALGX_BF16 && fast) ? 1 : 0, acc, (const TT*)q_src, gain_q, (const TT*)k_src,
                            gain_k, rope_cos, rope_sin, (int)T, (TT*)dq_out, (TT*)dk_out, partial, counter, dgain_q,
                            dgain_k, rows, eps, (int)H, tok_stride, (const TT*)dq_h, (const TT*)dk_h,
                            (const TT*)(dv_out ? dv_h : nullptr), (TT*)dv_out);
  };
  ALGX_REQUIRE((tok_stride == 0) == (dv_out == nullptr), "qknorm_attn_bwd: the packed layout needs dv_out");
  if (dtype == ALGX_BF16)
    ALGX_CUDA(tok_stride ? launch(__nv_bfloat16{}, std::true_type{}) : launch(__nv_bfloat16{}, std::false_type{}));
  else
    ALGX_CUDA(tok_stride ? launch(float{}, std::true_type{}) : launch(float{}, std::false_type{}));
  ALGX_LAUNCHED("qknorm_attn_bwd launch");
  return ALGX_OK;
}

size_t packed_scratch_off(int64_t B, int64_t H, int64_t T, int64_t D) {
  return align256(algx_qknorm_attn_bwd_workspace_size(B, H, T, D));
}
size_t packed_scratch_bytes(int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype) {
  return align256((size_t)B * H * T * D * (dtype == ALGX_BF16 ? 2 : 4));
}
}  // namespace
}  // namespace algx

extern "C" {

int algx_qknorm_attn_bwd(const algx_attn_config* cfg, const void* q, const void* k, const float* gain_q,
                         const float* gain_k, const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                         const void* q_scaled, const void* k_norm, const void* v,
                         const float* sink, const float* guard, const void* o, const float* o_precise,
                         const float* stat, const void* dout, void* dq, void* dk, void* dv, float* dgain_q,
                         float* dgain_k, float* dsink, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                         float eps, void* workspace, size_t workspace_bytes, void* stream) {
  return qknorm_attn_bwd_impl(cfg, q, k, gain_q, gain_k, rope_cos, rope_sin, rope_rows, q_scaled, k_norm, v, sink,
                              guard, o, o_precise, stat, dout, dq, dk, dv, dq, dk, nullptr, 0, dgain_q, dgain_k, dsink,
                              B, H, T, D, dtype, eps, workspace, workspace_bytes, stream);
}

size_t algx_qknorm_attn_bwd_packed_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype) {
  return packed_scratch_off(B, H, T, D) + 3 * packed_scratch_bytes(B, H, T, D, dtype);
}

int algx_qknorm_attn_bwd_packed(const algx_attn_config* cfg, const void* qkv, const float* gain_q,
                                const float* gain_k, const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                                const void* q_scaled, const void* k_norm, const void* v_heads, const float* sink,
                                const float* guard, const void* o, const float* o_precise, const float* stat,
                                const void* dout, void* dqkv, float* dgain_q, float* dgain_k, float* dsink,
                                int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype, float eps,
                                void* workspace, size_t workspace_bytes, void* stream) {
  ALGX_REQUIRE(qkv && dqkv, "qknorm_attn_bwd_packed: NULL pointer");
  ALGX_REQUIRE(H > 0 && 3 * H <= INT32_MAX, "qknorm_attn_bwd_packed: bad head count");
  ALGX_REQUIRE(B >= 0 && T > 0 && B * H * T <= INT32_MAX, "qknorm_attn_bwd_packed: B*H*T must be below 2^31");
  ALGX_REQUIRE(workspace && workspace_bytes >= algx_qknorm_attn_bwd_packed_workspace_size(B, H, T, D, dtype),
               "qknorm_attn_bwd_packed: workspace too small (see algx_qknorm_attn_bwd_packed_workspace_size)");
  const size_t es = dtype == ALGX_BF16 ? 2 : 4;
  const size_t blk = (size_t)H * (size_t)D * es;
  const char* in = static_cast<const char*>(qkv);
  char* out = static_cast<char*>(dqkv);
  char* scratch = static_cast<char*>(workspace) + packed_scratch_off(B, H, T, D);
  const size_t sb = packed_scratch_bytes(B, H, T, D, dtype);
  return qknorm_attn_bwd_impl(cfg, in, in + blk, gain_q, gain_k, rope_cos, rope_sin, rope_rows, q_scaled, k_norm,
                              v_heads, sink, guard, o, o_precise, stat, dout, scratch, scratch + sb, scratch + 2 * sb,
                              out, out + blk, out + 2 * blk, (int)(3 * H), dgain_q, dgain_k, dsink, B, H, T, D, dtype,
                              eps, workspace, workspace_bytes, stream);
}

}  // extern "C"
