// tcgen05 attention fast path: bf16 I/O, D = 64, T % 128 == 0, asinh with
// fast rho, n in {8, 16, 32}: the unshifted branch (the guarded low branch or
// the explicit clipped link) and the range guard's shifted high branch.
//
// Forward (kernels/flash.py:189-284, head_resident.py:24-93): one CTA per
// (128-query tile, head), two CTAs per SM. Warp roles: warps 0-7 compute the
// weights in two groups (thread = query row = TMEM lane), warp 8 issues TMA
// loads, warps 9 and 10 issue the tcgen05 MMAs (O += P V and S = Q K^T). S = Q K^T lands in TMEM (fp32), the weight warps turn
// each row into p = rho(x)^n, accumulate the fp32 row sum, and write bf16 P
// back into TMEM; O += P V reads P from TMEM (A operand) and V from shared
// memory (MN-major). No running maximum exists on this branch, so O needs no
// rescaling; O = acc / l and stat = 1/l (or l^(-1/n)) at the end. The shifted
// branch takes the row maximum in a first pass over the keys (see below).
//
// Backward (kernels/flash.py:333-361, 435-627): one CTA per (128-key tile,
// head). K, V stay resident; Q, dO, stat and di stream through a 4-stage TMA
// ring of 64-query halves, each released as soon as its sub-tile's products
// have read it.
// Per query tile: S^T = K Q^T and dP^T = V dO^T in TMEM; the score-gradient
// warps (thread = key row) recompute p = rho^n * stat, ds = p (dp - di) r,
// write bf16 P^T and dS^T to shared memory (128-byte swizzled K-major); then
// dV += P^T dO, dK += dS^T Q, and dQ_tile = dS K (the same dS^T buffer read
// MN-major). The score gradients are computed by two groups of eight warps
// that take alternate 64-query sub-tiles, so one sub-tile's stores and
// barrier round trips overlap the next one's arithmetic. A thread waits ~100
// cycles per tcgen05.mma it issues, so the three groups of products are
// issued by three threads that keep the tensor pipe fed in parallel.
// dQ_tile alternates between two TMEM buffers; warps 8-11 drain it into a
// 128-byte-swizzled fp32 staging tile in shared memory, from which one thread
// adds it to the fp32 accumulator in global memory with two TMA reduce-adds
// (the reduction runs in L2, off the SM's load/store path). A final pass
// scales and rounds the accumulator. Every mbarrier wait is bounded
// (sm100.cuh).
#include <algorithm>

#include "attn_common.cuh"
#include "attn_tc.h"
#include "sm100.cuh"
#include "tmap.h"

namespace algx {
namespace {

using namespace sm100;

constexpr int kTile = 128;
constexpr int kTileBytes = kTile * 64 * 2;  // 128 rows x 64 bf16
constexpr int kFwdKStages = 3;  // S = Q K^T runs up to three sub-tiles ahead of P.V ...
constexpr int kFwdVStages = 2;  // ... so K tiles are needed earlier than V tiles
constexpr int kFwdThreads = 352;  // 8 weight warps, producer, P.V issuer, S issuer
constexpr int kFwdProducer = 8;
constexpr int kFwdSmem = kTileBytes * (1 + kFwdKStages + kFwdVStages) + 1024;
constexpr int kBwdThreads = 800;
constexpr int kHalfBytes = kTileBytes / 2;  // 64 rows x 64 bf16
constexpr int kBwdStages = 4;               // Q / dO ring of 64-query halves
// K x2, V, the Q / dO ring, dS^T x2 tiles, dQ boxes x2, stat / di, alignment slack
constexpr int kBwdSmem = 3 * kTileBytes + 2 * kBwdStages * kHalfBytes + 4 * kTileBytes + 2 * kTileBytes +
                         2 * kBwdStages * 64 * 4 + 1024;
constexpr int kBwdGradWarps = 16, kBwdDrain = 16, kBwdProducer = 20;


__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// One asinh weight on the unshifted branch: rho(min(x, clamp))^N (fast rho).
template <int N, bool CLIP>
__device__ __forceinline__ float weight(float x, float clamp, float& r) {
  if constexpr (CLIP) x = fminf(x, clamp);
  const float rad = fmaf(x, x, 1.f);
  r = rsqrtf(rad);
  return ipow_t<N>(fmaf(rad, r, x));
}

// Weights of 32 scores of one row (one TMEM chunk): p = rho(x)^N with the
// fast radical, packed to bf16 pairs for the P.V MMA; returns the fp32 sum.
// DIAG masks keys after the query (col > r) on the diagonal tile only.
template <int N, bool CLIP, bool DIAG>
__device__ __forceinline__ float weights_chunk(const uint32_t (&sv)[32], uint32_t (&pk)[16], float clamp, int col0,
                                               int r) {
  const float2 one = make_float2(1.f, 1.f);
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float2 x = make_float2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
    if constexpr (CLIP) {
      x.x = fminf(x.x, clamp);
      x.y = fminf(x.y, clamp);
    }
    const float2 rad = fma2(x, x, one);
    const float2 rr = make_float2(rsqrt_fast(rad.x), rsqrt_fast(rad.y));
    float2 p = ipow2_t<N>(fma2(rad, rr, x));
    if constexpr (DIAG) {
      if (col0 + 2 * i > r) p.x = 0.f;
      if (col0 + 2 * i + 1 > r) p.y = 0.f;
    }
    acc = add2(acc, p);
    pk[i] = pack_bf16x2(p.x, p.y);
  }
  return acc.x + acc.y;
}

// p and ds (without the slope n) of C scores of one key row against C query
// columns (kernels/flash.py:333-361), packed to bf16 pairs. EXACT: the stable
// rho of the shifted branch, 1 / (|x| + sqrt(1 + x^2)) for x < 0
// (kernels/flash.py:76-80), with the reciprocal on the MUFU pipe.
template <int N, bool CLIP, bool INV, bool DIAG, int C, bool EXACT = false>
__device__ __forceinline__ void grads_chunk(const uint32_t (&sv)[C], const uint32_t (&pv)[C],
                                            const float* __restrict__ st, const float* __restrict__ dd,
                                            uint32_t (&pk)[C / 2], uint32_t (&dk)[C / 2], float clamp, int col0,
                                            int r) {
  const float2 one = make_float2(1.f, 1.f);
#pragma unroll
  for (int i4 = 0; i4 < C / 4; ++i4) {
    const float4 s4 = *reinterpret_cast<const float4*>(st + 4 * i4);
    const float4 d4 = *reinterpret_cast<const float4*>(dd + 4 * i4);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = 2 * i4 + h;
      const float2 sc = make_float2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
      float2 x = sc;
      if constexpr (CLIP) {
        x.x = fminf(x.x, clamp);
        x.y = fminf(x.y, clamp);
      }
      const float2 rad = fma2(x, x, one);
      const float2 rr = make_float2(rsqrt_fast(rad.x), rsqrt_fast(rad.y));
      float2 rho;
      if constexpr (EXACT) {
        const float2 t = fma2(rad, rr, make_float2(fabsf(x.x), fabsf(x.y)));
        rho.x = x.x >= 0.f ? t.x : rcp_fast(t.x);
        rho.y = x.y >= 0.f ? t.y : rcp_fast(t.y);
      } else {
        rho = fma2(rad, rr, x);
      }
      const float2 stc = h ? make_float2(s4.z, s4.w) : make_float2(s4.x, s4.y);
      const float2 dic = h ? make_float2(d4.z, d4.w) : make_float2(d4.x, d4.y);
      float2 p = INV ? mul2(ipow2_t<N>(rho), stc) : ipow2_t<N>(mul2(rho, stc));
      const float2 dpv = make_float2(__uint_as_float(pv[2 * i]), __uint_as_float(pv[2 * i + 1]));
      float2 ds = mul2(mul2(p, sub2(dpv, dic)), rr);
      if constexpr (CLIP) {
        if (!(sc.x < clamp)) ds.x = 0.f;
        if (!(sc.y < clamp)) ds.y = 0.f;
      }
      if constexpr (DIAG) {
        if (col0 + 2 * i < r) p.x = ds.x = 0.f;
        if (col0 + 2 * i + 1 < r) p.y = ds.y = 0.f;
      }
      pk[i] = pack_bf16x2(p.x, p.y);
      dk[i] = pack_bf16x2(ds.x, ds.y);
    }
  }
}

// ---------------------------------------------------------------- forward
// The key loop runs over 64-key sub-tiles u = 2j + h of the 128-key TMA
// tiles j. TMEM (256 columns): three score buffers B[u % 3] = base + 64(u % 3)
// (fp32, 128 x 64) and O = base + 192 (fp32, 128 x 64). The weight warps read
// S_u into registers and write the bf16 P_u into the first 32 columns of the
// same buffer; O += P_u V reads it there. S and P.V are issued by two
// threads (a thread waits ~100 cycles per tcgen05.mma it issues); the S
// thread runs up to three sub-tiles ahead: S_{u+3} goes into buffer u % 3 as
// soon as P_u.V has completed. Two groups of four weight warps take alternate sub-tiles (each
// warp: its 32 query rows, the sub-tile's 64 keys in two 32-column chunks),
// so one group's TMEM round trips and barrier waits overlap the other's
// arithmetic; their partial row sums meet in shared memory at the end.
//
// Shifted branch (range guard's high branch, kernels/flash.py:200-214,
// 246-259): the weights are (rho(x) / rho(m))^n with m the row maximum of the
// scores (and the sink logit). Rather than rescaling O in TMEM whenever a
// running maximum grows, the body makes two passes over the keys: pass A
// computes S = Q K^T only and takes the exact row maximum, pass B computes
// the weights against that fixed m, so O and l accumulate without any
// rescale. The result is the reference's up to rounding (a common factor of
// every weight cancels in O / l). The sub-tile counter runs over both passes
// (2 x nu sub-tiles), so every barrier keeps one phase sequence; pass A's
// sub-tiles are released by the P.V thread without a product.

// Weights of 32 scores of one row on the shifted branch: p = (rho(x) * shift)^N
// with the stable rho (1 / (|x| + sqrt(1 + x^2)) for x < 0, kernels/flash.py:76-80)
// and shift = 1 / rho(m); returns the fp32 sum.
template <int N, bool DIAG>
__device__ __forceinline__ float weights_chunk_shifted(const uint32_t (&sv)[32], uint32_t (&pk)[16], float shift,
                                                       int col0, int r) {
  const float2 one = make_float2(1.f, 1.f), sh = make_float2(shift, shift);
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = make_float2(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1]));
    const float2 rad = fma2(x, x, one);
    const float2 rr = make_float2(rsqrt_fast(rad.x), rsqrt_fast(rad.y));
    const float2 t = fma2(rad, rr, make_float2(fabsf(x.x), fabsf(x.y)));
    float2 rho;
    rho.x = x.x >= 0.f ? t.x : rcp_fast(t.x);
    rho.y = x.y >= 0.f ? t.y : rcp_fast(t.y);
    float2 p = ipow2_t<N>(mul2(rho, sh));
    if constexpr (DIAG) {
      if (col0 + 2 * i > r) p.x = 0.f;
      if (col0 + 2 * i + 1 > r) p.y = 0.f;
    }
    acc = add2(acc, p);
    pk[i] = pack_bf16x2(p.x, p.y);
  }
  return acc.x + acc.y;
}

// Row maximum of 32 scores (keys after the query excluded on the diagonal).
template <bool DIAG>
__device__ __forceinline__ float max_chunk(const uint32_t (&sv)[32], float m, int col0, int r) {
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (!DIAG || col0 + i <= r) m = fmaxf(m, __uint_as_float(sv[i]));
  return m;
}

template <int N, bool CLIP, bool SHIFTED>
__device__ __forceinline__ void attn_fwd_tc_body(const CUtensorMap* tq, const CUtensorMap* tk, const CUtensorMap* tv,
                                                 const algx_attn_config& cfg, const float* __restrict__ sink,
                                                 const Eff& e, __nv_bfloat16* __restrict__ o,
                                                 float* __restrict__ o_prec, float* __restrict__ stat, int H, int T,
                                                 int* dev_err) {
  constexpr int kPasses = SHIFTED ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;
  uint8_t* sV = sK + kFwdKStages * kTileBytes;
  __shared__ uint64_t bar_q, bar_o_full, bar_l_ready, bar_s_full[3], bar_p_full[3], bar_p_free[3], bar_issued[2];
  __shared__ uint64_t bar_k_full[kFwdKStages], bar_k_empty[kFwdKStages], bar_v_full[kFwdVStages],
      bar_v_empty[kFwdVStages];
  __shared__ float l_part[kTile];  // row sums of weight group 1
  __shared__ float m_part[SHIFTED ? 2 * kTile : 1];  // pass A row maxima of the two groups
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;

  // warps 0-7: weights (group g = warp / 4 takes sub-tiles u % 2 == g; rows 32 (warp % 4)..)
  // warp 8: TMA producer (+ TMEM owner); warp 9: O += P V issuer; warp 10: S = Q K^T issuer
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = T / kTile;
  // The scheduler dispatches blockIdx.x fastest: heads along x and the query
  // tile along y (reversed) start every head's longest rows first.
  const int qt = nq - 1 - (int)blockIdx.y;
  const int bh = blockIdx.x;
  const int nk = qt + 1;   // 128-key tiles
  const int nu = 2 * nk;   // 64-key sub-tiles of one pass
  const int row_base = bh * T;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_o_full, 1);
    mbar_init(&bar_l_ready, 4);
    mbar_init(&bar_issued[0], 1);
    mbar_init(&bar_issued[1], 1);
    for (int b = 0; b < 3; ++b) {
      mbar_init(&bar_s_full[b], 1);
      mbar_init(&bar_p_full[b], 4);  // the four warps of the group that owns the sub-tile
      mbar_init(&bar_p_free[b], 1);
    }
    for (int s = 0; s < kFwdKStages; ++s) {
      mbar_init(&bar_k_full[s], 1);
      mbar_init(&bar_k_empty[s], 1);
    }
    for (int s = 0; s < kFwdVStages; ++s) {
      mbar_init(&bar_v_full[s], 1);
      mbar_init(&bar_v_empty[s], 1);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == kFwdProducer) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = tmem_base, tO = tmem_base + 192;
  // Before the CTA frees TMEM, each issuer waits (bounded) until its own
  // products have completed, on the normal and on the abort path alike.
  auto settle_issuer = [&](int i) {
    mma_commit(&bar_issued[i]);
    volatile int quiet = 0;
    mbar_wait(&bar_issued[i], 0, &quiet, dev_err);
  };

  if (warp == kFwdProducer) {
    if (lane == 0) {
      prefetch_tmap(tq);
      prefetch_tmap(tk);
      prefetch_tmap(tv);
      mbar_expect_tx(&bar_q, kTileBytes);
      tma_load_2d(sQ, tq, &bar_q, 0, row_base + qt * kTile);
      // K load J (tile J % nk), then V tile j of the weighted pass: K waits
      // for the S products of load J - 3, V for the P.V products of tile j - 2.
      int issued_k[kFwdKStages] = {-1, -1, -1}, issued_v[kFwdVStages] = {-1, -1};
      for (int J = 0; J < kPasses * nk; ++J) {
        const int sk = J % kFwdKStages;
        if (J >= kFwdKStages && !mbar_wait(&bar_k_empty[sk], ((J / kFwdKStages) - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&bar_k_full[sk], kTileBytes);
        tma_load_2d(sK + sk * kTileBytes, tk, &bar_k_full[sk], 0, row_base + (J % nk) * kTile);
        issued_k[sk] = J;
        if (SHIFTED && J < nk) continue;  // pass A reads no V
        const int j = SHIFTED ? J - nk : J, sv = j % kFwdVStages;
        if (j >= kFwdVStages && !mbar_wait(&bar_v_empty[sv], ((j / kFwdVStages) - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&bar_v_full[sv], kTileBytes);
        tma_load_2d(sV + sv * kTileBytes, tv, &bar_v_full[sv], 0, row_base + j * kTile);
        issued_v[sv] = j;
      }
      if (*abort_v) {  // let copies in flight land before the CTA exits
        volatile int quiet = 0;
        for (int s = 0; s < kFwdKStages; ++s)
          if (issued_k[s] >= 0) mbar_wait(&bar_k_full[s], (issued_k[s] / kFwdKStages) & 1, &quiet, nullptr);
        for (int s = 0; s < kFwdVStages; ++s)
          if (issued_v[s] >= 0) mbar_wait(&bar_v_full[s], (issued_v[s] / kFwdVStages) & 1, &quiet, nullptr);
      }
    }
  } else if (warp == kFwdProducer + 2) {
    // ----- S_w = Q K_J^T into buffer w % 3 (K rows of half w & 1 of load J = w >> 1),
    // up to three sub-tiles ahead of the P.V products
    if (lane == 0) {
      const uint32_t idS = idesc_bf16_f32(128, 64, 0, 0);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK);
      bool ok = mbar_wait(&bar_q, 0, abort_v, dev_err);
      for (int w = 0; ok && w < kPasses * nu; ++w) {
        const int b = w % 3, J = w >> 1, s = J % kFwdKStages;
        if ((w & 1) == 0 && !mbar_wait(&bar_k_full[s], (J / kFwdKStages) & 1, abort_v, dev_err)) break;
        if (w >= 3 && !mbar_wait(&bar_p_free[b], (w / 3 - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t kb = k0 + s * kTileBytes + (w & 1) * (kTileBytes / 2);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_ss(tS + 64 * b, desc_sw128(q0 + k * 32, 16, 1024), desc_sw128(kb + k * 32, 16, 1024), idS, k > 0);
        mma_commit(&bar_s_full[b]);
        if (w & 1) mma_commit(&bar_k_empty[s]);  // both halves of K load J have been read
      }
      settle_issuer(0);
    }
  } else if (warp == kFwdProducer + 1) {
    // ----- O += P_u V_u, P_u in the first 32 columns of buffer u % 3; the
    // commit after P.V of a tile's second half releases its V stage. Pass A
    // sub-tiles only hand their buffer back once the weight warps have read it.
    if (lane == 0) {
      const uint32_t idO = idesc_bf16_f32(128, 64, 0, 1);
      const uint32_t v0 = smem_u32(sV);
      for (int w = 0; w < kPasses * nu; ++w) {
        const int b = w % 3;
        if (!mbar_wait(&bar_p_full[b], (w / 3) & 1, abort_v, dev_err)) break;
        if (SHIFTED && w < nu) {
          mbar_arrive(&bar_p_free[b]);
          continue;
        }
        const int u = SHIFTED ? w - nu : w, j = u >> 1, s = j % kFwdVStages;
        if ((u & 1) == 0 && !mbar_wait(&bar_v_full[s], (j / kFwdVStages) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t vb = v0 + s * kTileBytes + (u & 1) * (kTileBytes / 2);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_ts(tO, tS + 64 * b + k * 8, desc_sw128(vb + k * 2048, 8192, 1024), idO, (u > 0 || k > 0));
        mma_commit(&bar_p_free[b]);
        if (u & 1) mma_commit(&bar_v_empty[s]);
        if (u == nu - 1) mma_commit(&bar_o_full);
      }
      settle_issuer(1);
    }
  } else {
    // ----- weight warps: thread r owns query row qt*128 + r (TMEM lane r)
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float l = 0.f, rr, shift = 1.f;
    bool ok = true;
    int w0 = g;  // first sub-tile of the weighted pass owned by this group
    if constexpr (SHIFTED) {
      // pass A: the row maximum over the causal keys
      float m = -INFINITY;
      for (int u = g; u < nu; u += 2) {
        const int b = u % 3;
        if (!mbar_wait_warp(&bar_s_full[b], (u / 3) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
        const bool diag = (u >> 1) == qt;
        const int col0 = 64 * (u & 1);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tc_fence_after();
          uint32_t sv[32];
          tmem_ld32(tS + 64 * b + 32 * c + lane_off, sv);
          m = diag ? max_chunk<true>(sv, m, col0 + 32 * c, r) : max_chunk<false>(sv, m, col0 + 32 * c, r);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_p_full[b]);
      }
      // both groups meet here once, also after an aborted wait (every one of
      // the 256 threads reaches this barrier exactly once)
      m_part[g * kTile + r] = m;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      m = fmaxf(m_part[r], m_part[kTile + r]);
      if (cfg.has_sink) m = fmaxf(m, sink[bh % H]);
      shift = rho_exact(-m, rr);  // 1 / rho(m)
      if (g == 0 && cfg.has_sink) l = ipow_t<N>(rho_exact(sink[bh % H], rr) * shift);
      w0 = nu + g;
    } else {
      if (g == 0 && cfg.has_sink) l = weight<N, CLIP>(sink[bh % H], cfg.clamp, rr);
    }
    for (int w = w0; ok && w < kPasses * nu; w += 2) {
      const int b = w % 3, u = SHIFTED ? w - nu : w;
      if (!mbar_wait_warp(&bar_s_full[b], (w / 3) & 1, abort_v, dev_err)) {
        ok = false;
        break;
      }
      const bool diag = (u >> 1) == qt;
      const int col0 = 64 * (u & 1);  // key offset within the 128-key tile
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tc_fence_after();
        uint32_t sv[32], pk[16];
        tmem_ld32(tS + 64 * b + 32 * c + lane_off, sv);
        if constexpr (SHIFTED) {
          if (diag)
            l += weights_chunk_shifted<N, true>(sv, pk, shift, col0 + 32 * c, r);
          else
            l += weights_chunk_shifted<N, false>(sv, pk, shift, col0 + 32 * c, r);
        } else {
          if (diag)
            l += weights_chunk<N, CLIP, true>(sv, pk, cfg.clamp, col0 + 32 * c, r);
          else
            l += weights_chunk<N, CLIP, false>(sv, pk, cfg.clamp, col0 + 32 * c, r);
        }
        // P (bf16 pairs) over S columns 16c..16c+15, already consumed by this thread
        tmem_st16(tS + 64 * b + 16 * c + lane_off, pk);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p_full[b]);
    }
    if (g == 1) {
      l_part[r] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_l_ready);  // release: l_part is visible to group 0
    } else if (ok && mbar_wait_warp(&bar_l_ready, 0, abort_v, dev_err) &&
               mbar_wait_warp(&bar_o_full, 0, abort_v, dev_err)) {
      tc_fence_after();
      l += l_part[r];
      const float inv = 1.f / l;
      const size_t row = (size_t)row_base + (size_t)qt * kTile + r;
      uint4* dst = reinterpret_cast<uint4*>(o + row * 64);
      float4* dst_prec = reinterpret_cast<float4*>(o_prec + (SHIFTED ? row * 64 : 0));
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t ov[32];
        tmem_ld32(tO + lane_off + 32 * c, ov);
#pragma unroll
        for (int un = 0; un < 4; ++un) {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(ov[8 * un + i]) * inv;
          uint4 w;
          w.x = pack_bf16x2(f[0], f[1]);
          w.y = pack_bf16x2(f[2], f[3]);
          w.z = pack_bf16x2(f[4], f[5]);
          w.w = pack_bf16x2(f[6], f[7]);
          dst[c * 4 + un] = w;
          if constexpr (SHIFTED) {  // the unrounded output (kernels/flash.py:851-852)
            dst_prec[c * 8 + 2 * un] = make_float4(f[0], f[1], f[2], f[3]);
            dst_prec[c * 8 + 2 * un + 1] = make_float4(f[4], f[5], f[6], f[7]);
          }
        }
      }
      if constexpr (SHIFTED)
        stat[row] = shift * inv_root(l, N);  // 1 / (rho(m) l^(1/n))
      else
        stat[row] = e.inv_stat ? inv : inv_root(l, N);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kFwdProducer) tmem_dealloc(tmem_base, 256);
}

// The unshifted body always; with the range guard (CLIP false) also the
// shifted one, chosen on the device from the prologue's maxima, so neither
// branch needs a second launch.
template <int N, bool CLIP>
__global__ void __launch_bounds__(kFwdThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, algx_attn_config cfg, const float* __restrict__ sink,
                       const float* __restrict__ guard, __nv_bfloat16* __restrict__ o, float* __restrict__ o_prec,
                       float* __restrict__ stat, int H, int T, int* dev_err) {
  pdl_wait();  // launched as a dependent of the prologue, which writes q_scaled and the guard maxima
  const Eff e = resolve_variant(cfg, guard);
  // No early launch_dependents: this grid runs in several waves (two CTAs per
  // SM), and a dependent launched now would hold SMs its later waves need while
  // it waits (measured: 8 us of the config-2 step).
  if (e.branch == BR_UNSHIFTED) {
    attn_fwd_tc_body<N, CLIP, false>(&tq, &tk, &tv, cfg, sink, e, o, o_prec, stat, H, T, dev_err);
  } else if constexpr (!CLIP) {
    if (e.branch == BR_SHIFTED && cfg.mode == ALGX_MODE_GUARDED)
      attn_fwd_tc_body<N, false, true>(&tq, &tk, &tv, cfg, sink, e, o, o_prec, stat, H, T, dev_err);
  }
}

// ---------------------------------------------------------------- backward
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Byte offset of bf16 element (row, col) in a [128 rows][128 cols] tile kept
// as two 128-byte-swizzled K-major halves of 64 columns.
__device__ __forceinline__ uint32_t sw128_off(int row, int col16) {
  // col16: index of the 16-byte unit (8 bf16) in [0, 16)
  const int half = col16 >> 3, u = col16 & 7;
  return half * kTileBytes + row * 128 + ((u ^ (row & 7)) << 4);
}

// One work item of the persistent backward: key tile kt of head bh. Items
// are handed out heaviest first (kt ascending: key tile kt meets nq - kt
// query tiles) through a global counter, so SMs that finish early take the
// next largest remaining item.
struct BwdItem {
  int kt, bh, ni;  // ni query tiles, 2 * ni sub-tiles
};
__device__ __forceinline__ BwdItem bwd_item(int it, int BH, int nq) {
  BwdItem r;
  r.kt = it / BH;
  r.bh = it - r.kt * BH;
  r.ni = nq - r.kt;
  return r;
}

// Persistent backward: one CTA per SM walks work items. Per item, the
// 64-query sub-tiles u = 2*ii + h of its query tiles ii (h = u & 1 is also
// the TMEM buffer) run through the pipeline below; every ring and barrier
// is indexed by counters that continue across items, so the next item's
// loads and products overlap the end of the current one.
// TMEM (512 columns): S^T[b] = base + 64b, dP^T[b] = base + 128 + 64b (fp32,
// 128 keys x 64 queries), dV = base + 256, dK = base + 320, dQ_tile = base +
// 384, P^T[b] = base + 448 + 32b (bf16 pairs: the A operand of dV += P^T dO).
// Shared memory: K double-buffered (S^T and the dQ products of an item read
// it), V, a 4-stage ring of 64-query Q / dO / stat / di halves, dS^T of two
// query tiles (each two 128B-swizzled 64-column halves side by side: exactly
// the MN-major A operand of dQ_tile = dS K), and two 16 KB fp32 staging
// boxes for the dQ reduce-adds.
// SHIFTED: the instantiation for the range guard's shifted (high) branch:
// exact rho, root statistic (p = (rho * stat)^N, kernels/flash.py:246-259),
// no clamp; it runs only when the guard chose that branch, the unshifted
// instantiation only when it did not.
template <int N, bool CLIP, bool INV_STAT, bool SHIFTED = false>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                       const __grid_constant__ CUtensorMap tdq, const __grid_constant__ CUtensorMap tdk,
                       const __grid_constant__ CUtensorMap tdv, algx_attn_config cfg, const float* __restrict__ stat,
                       const float* __restrict__ di, const float* __restrict__ guard, int* __restrict__ item_counter,
                       int BH, int T, int* dev_err) {
  pdl_wait();  // launched as a dependent of the di pass, which writes di and zeroes the accumulator
  const Eff e = resolve_variant(cfg, guard);
  if (e.branch != (SHIFTED ? BR_SHIFTED : BR_UNSHIFTED)) return;
  pdl_trigger();  // the fallback kernels may be scheduled behind this grid
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sK = smem;                     // 2 buffers
  uint8_t* sV = smem + 2 * kTileBytes;
  uint8_t* sQ = smem + 3 * kTileBytes;    // kBwdStages x 64 queries
  uint8_t* sdO = sQ + kBwdStages * kHalfBytes;
  uint8_t* sdST = sdO + kBwdStages * kHalfBytes;  // 128 keys x 128 queries bf16, [2 query tiles][2 halves]
  uint8_t* sDQ = sdST + 4 * kTileBytes;           // fp32 dQ staging: two 128-row x 32-column swizzled boxes
  float* sStat = reinterpret_cast<float*>(sDQ + 2 * kTileBytes);  // [kBwdStages][64]
  float* sDi = sStat + kBwdStages * 64;                              // [kBwdStages][64]
  __shared__ uint64_t bar_k_full[2], bar_k_free[2], bar_v_full, bar_v_free, bar_fin, bar_acc_free;
  __shared__ uint64_t bar_dq_full, bar_dq_free, bar_stage_full[2], bar_stage_free[2];
  __shared__ uint64_t bar_st_full[2], bar_st_free[2], bar_ps_ready[2], bar_p_free[2], bar_ds_free[2], bar_ds_ready[2];
  __shared__ uint64_t bar_qd_full[kBwdStages], bar_qd_empty[kBwdStages], bar_issued[4];
  __shared__ uint64_t bar_item_full[4], bar_item_empty[4];
  __shared__ int item_q[4];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  volatile int* item_v = item_q;
  // Before the CTA frees TMEM, each issuer waits (bounded) until its own
  // products have completed, on the normal and on the abort path alike.
  auto settle_issuer = [&](int i) {
    mma_commit(&bar_issued[i]);
    volatile int quiet = 0;
    mbar_wait(&bar_issued[i], 0, &quiet, dev_err);
  };
  // Consumers of the item queue: one arrival per consumer warp on
  // bar_item_empty (16 gradient + 4 drain warps + 4 issuers).
  constexpr int kItemConsumers = kBwdGradWarps + 4 + 4;
  auto next_item = [&](int j, bool whole_warp) -> int {
    const int slot = j & 3;
    bool ok = whole_warp ? mbar_wait_warp(&bar_item_full[slot], (j >> 2) & 1, abort_v, dev_err)
                         : mbar_wait(&bar_item_full[slot], (j >> 2) & 1, abort_v, dev_err);
    const int it = ok ? item_v[slot] : -1;
    if (whole_warp) __syncwarp();
    if (!whole_warp || (threadIdx.x & 31) == 0) mbar_arrive(&bar_item_empty[slot]);
    return it;
  };

  // warps 0-15: score gradients; warp w takes the sub-tiles u with u % 2 == w / 8 (TMEM buffer w / 8),
  //   TMEM lanes 32 (w % 4).. and query columns 32 ((w / 4) % 2).. of each
  // warps 16-19: dQ drain and the dK / dV write-out; warp 20: item queue + TMA producer (+ TMEM owner);
  // warps 21-24: MMA issuers (21: S^T, 22: dV and dK, 23: dQ, 24: dP^T). A
  // thread spends ~100 cycles issuing one tcgen05.mma, so S^T and dP^T of the
  // next sub-tile come from two threads in parallel.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = T / kTile;
  const int total_items = BH * nq;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_k_full[b], 1);
      mbar_init(&bar_k_free[b], 1);
      mbar_init(&bar_st_full[b], 2);  // S^T and dP^T issuers
      mbar_init(&bar_st_free[b], 8);
      mbar_init(&bar_ps_ready[b], 8);
      mbar_init(&bar_p_free[b], 1);
      mbar_init(&bar_ds_free[b], 1);
      mbar_init(&bar_ds_ready[b], 16);  // 8 gradient warps x 2 sub-tiles of a query tile
    }
    for (int i = 0; i < kBwdStages; ++i) {
      mbar_init(&bar_qd_full[i], 1);
      mbar_init(&bar_qd_empty[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar_item_full[i], 1);
      mbar_init(&bar_item_empty[i], kItemConsumers);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&bar_issued[i], 1);
    mbar_init(&bar_v_full, 1);
    mbar_init(&bar_v_free, 1);
    mbar_init(&bar_fin, 1);
    mbar_init(&bar_acc_free, 4);
    mbar_init(&bar_dq_full, 1);
    mbar_init(&bar_dq_free, 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_stage_full[b], 4);
      mbar_init(&bar_stage_free[b], 1);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == kBwdProducer) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = tmem_base, tdP = tmem_base + 128, tdV = tmem_base + 256, tdK = tmem_base + 320,
                 tdQ = tmem_base + 384, tPT = tmem_base + 448;

  if (warp == kBwdProducer) {
    // ----- item queue and TMA producer
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&tdo);
      prefetch_tmap(&tdq);
      prefetch_tmap(&tdk);
      prefetch_tmap(&tdv);
      int pending_k[2] = {-1, -1}, pending_v = -1, pending_qd[kBwdStages] = {-1, -1, -1, -1};
      int U = 0;  // global sub-tile counter
      for (int j = 0;; ++j) {
        const int slot = j & 3;
        if (j >= 4 && !mbar_wait(&bar_item_empty[slot], ((j >> 2) - 1) & 1, abort_v, dev_err)) break;
        int it = atomicAdd(item_counter, 1);
        if (it >= total_items) it = -1;
        item_v[slot] = it;
        mbar_arrive(&bar_item_full[slot]);  // release: the item index is visible to the waiters
        if (it < 0) break;
        const BwdItem w = bwd_item(it, BH, nq);
        const int row_base = w.bh * T;
        const int kb = j & 1;
        if (j >= 2 && !mbar_wait(&bar_k_free[kb], ((j >> 1) - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&bar_k_full[kb], kTileBytes);
        tma_load_2d(sK + kb * kTileBytes, &tk, &bar_k_full[kb], 0, row_base + w.kt * kTile);
        pending_k[kb] = j;
        if (j >= 1 && !mbar_wait(&bar_v_free, (j - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&bar_v_full, kTileBytes);
        tma_load_2d(sV, &tv, &bar_v_full, 0, row_base + w.kt * kTile);
        pending_v = j;
        bool ok = true;
        for (int u = 0; u < 2 * w.ni; ++u, ++U) {
          const int hs = U % kBwdStages;
          const int q_row = row_base + (w.kt + (u >> 1)) * kTile + 64 * (u & 1);
          if (U >= kBwdStages && !mbar_wait(&bar_qd_empty[hs], ((U / kBwdStages) - 1) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bar_qd_full[hs], 2 * kHalfBytes + 2 * 64 * 4);
          tma_load_2d(sQ + hs * kHalfBytes, &tq, &bar_qd_full[hs], 0, q_row);
          tma_load_2d(sdO + hs * kHalfBytes, &tdo, &bar_qd_full[hs], 0, q_row);
          bulk_load(sStat + hs * 64, stat + q_row, 64 * 4, &bar_qd_full[hs]);
          bulk_load(sDi + hs * 64, di + q_row, 64 * 4, &bar_qd_full[hs]);
          pending_qd[hs] = U;
        }
        if (!ok) break;
      }
      if (*abort_v) {  // let copies in flight land before the CTA exits
        volatile int quiet = 0;
        for (int b = 0; b < 2; ++b)
          if (pending_k[b] >= 0) mbar_wait(&bar_k_full[b], (pending_k[b] >> 1) & 1, &quiet, nullptr);
        if (pending_v >= 0) mbar_wait(&bar_v_full, pending_v & 1, &quiet, nullptr);
        for (int i = 0; i < kBwdStages; ++i)
          if (pending_qd[i] >= 0) mbar_wait(&bar_qd_full[i], (pending_qd[i] / kBwdStages) & 1, &quiet, nullptr);
      }
    }
  } else if (warp == kBwdProducer + 1 || warp == kBwdProducer + 4) {
    // ----- S^T = K Q^T (warp 21) or dP^T = V dO^T (warp 24) of sub-tile u into buffer u & 1
    if (lane == 0) {
      const bool dp = warp == kBwdProducer + 4;
      const uint32_t idS = idesc_bf16_f32(128, 64, 0, 0);
      const uint32_t a0 = smem_u32(dp ? sV : sK), b0 = smem_u32(dp ? sdO : sQ);
      const uint32_t tacc = dp ? tdP : tS;
      int U = 0;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int it = next_item(j, false);
        if (it < 0) break;
        const BwdItem w = bwd_item(it, BH, nq);
        const int kb = j & 1;
        ok = dp ? mbar_wait(&bar_v_full, j & 1, abort_v, dev_err)
                : mbar_wait(&bar_k_full[kb], (j >> 1) & 1, abort_v, dev_err);
        const uint32_t abase = dp ? a0 : a0 + kb * kTileBytes;  // K double-buffered, V single
        for (int u = 0; ok && u < 2 * w.ni; ++u, ++U) {
          const int b = U & 1, hs = U % kBwdStages;
          if (!mbar_wait(&bar_qd_full[hs], (U / kBwdStages) & 1, abort_v, dev_err)) ok = false;
          if (ok && U >= 2 && !mbar_wait(&bar_st_free[b], ((U >> 1) - 1) & 1, abort_v, dev_err)) ok = false;
          if (!ok) break;
          tc_fence_after();
          const uint32_t bb = b0 + hs * kHalfBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ss(tacc + 64 * b, desc_sw128(abase + k * 32, 16, 1024), desc_sw128(bb + k * 32, 16, 1024), idS,
                   k > 0);
          mma_commit(&bar_st_full[b]);
        }
        if (ok && dp) mma_commit(&bar_v_free);  // every dP^T of the item has read V
      }
      settle_issuer(dp ? 3 : 0);
    }
  } else if (warp == kBwdProducer + 2) {
    // ----- dV += P^T dO and dK += dS^T Q of sub-tile w. S^T and dP^T of the
    // sub-tile, the other readers of its Q/dO half-stage, completed before its
    // score gradients were ready, so the commit after dK releases the stage.
    if (lane == 0) {
      const uint32_t idKM = idesc_bf16_f32(128, 64, 0, 1);  // A K-major (smem or TMEM), B MN-major
      const uint32_t q0 = smem_u32(sQ), do0 = smem_u32(sdO), dsb = smem_u32(sdST);
      int U = 0, I = 0;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int it = next_item(j, false);
        if (it < 0) break;
        const BwdItem w = bwd_item(it, BH, nq);
        // the write-out of the previous item has read dK and dV out of TMEM
        if (j >= 1 && !mbar_wait(&bar_acc_free, (j - 1) & 1, abort_v, dev_err)) break;
        for (int u = 0; u < 2 * w.ni; ++u, ++U) {
          const int b = U & 1, hs = U % kBwdStages, s = (I + (u >> 1)) & 1;
          if (!mbar_wait(&bar_ps_ready[b], (U >> 1) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qb = q0 + hs * kHalfBytes;
          const uint32_t db = do0 + hs * kHalfBytes;
          const uint32_t ds0 = dsb + s * 2 * kTileBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ts(tdV, tPT + 32 * b + 8 * k, desc_sw128(db + k * 2048, 8192, 1024), idKM, (u > 0 || k > 0));
          mma_commit(&bar_p_free[b]);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ss(tdK, desc_sw128(ds0 + b * kTileBytes + k * 32, 16, 1024), desc_sw128(qb + k * 2048, 8192, 1024),
                   idKM, (u > 0 || k > 0));
          mma_commit(&bar_qd_empty[hs]);
        }
        I += w.ni;
        if (ok) mma_commit(&bar_fin);  // dK and dV of the item are complete
      }
      settle_issuer(1);
    }
  } else if (warp == kBwdProducer + 3) {
    // ----- dQ_tile = dS K of query tile i
    if (lane == 0) {
      const uint32_t idMM = idesc_bf16_f32(128, 64, 1, 1);  // A MN-major smem, B MN-major
      const uint32_t k0 = smem_u32(sK), dsb = smem_u32(sdST);
      int I = 0;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int it = next_item(j, false);
        if (it < 0) break;
        const BwdItem w = bwd_item(it, BH, nq);
        const int kb = j & 1;
        if (!mbar_wait(&bar_k_full[kb], (j >> 1) & 1, abort_v, dev_err)) break;
        const uint32_t kbase = k0 + kb * kTileBytes;
        for (int ii = 0; ii < w.ni; ++ii, ++I) {
          const int s = I & 1;
          if (!mbar_wait(&bar_ds_ready[s], (I >> 1) & 1, abort_v, dev_err) ||
              (I >= 1 && !mbar_wait(&bar_dq_free, (I - 1) & 1, abort_v, dev_err))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ds0 = dsb + s * 2 * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_ss(tdQ, desc_sw128(ds0 + k * 2048, kTileBytes, 1024), desc_sw128(kbase + k * 2048, 8192, 1024),
                   idMM, k > 0);
          mma_commit(&bar_dq_full);
          mma_commit(&bar_ds_free[s]);
        }
        if (ok) mma_commit(&bar_k_free[kb]);  // the item's last product that reads K
      }
      settle_issuer(2);
    }
  } else if (warp < kBwdGradWarps) {
    // ----- score-gradient warps: group g = warp / 8 takes global sub-tiles U with U % 2 == g
    const int g = warp >> 3, q4 = warp & 3, hc = (warp >> 2) & 1;
    const int r = q4 * 32 + lane;  // key row within the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const int b = g;  // TMEM S^T / dP^T buffer and P^T half of this group
    int U = 0, I = 0;
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int it = next_item(j, true);
      if (it < 0) break;
      const BwdItem w = bwd_item(it, BH, nq);
      const int nu = 2 * w.ni;
      for (int u = g; u < nu; u += 2) {
        const int Ug = U + u, ii = u >> 1, Ig = I + ii, s = Ig & 1;
        if (!mbar_wait_warp(&bar_st_full[b], (Ug >> 1) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int hs = Ug % kBwdStages;
        uint32_t pk[2][8], dk2[2][8];
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          uint32_t sv[16], pv[16];
          const uint32_t col = 64 * b + 32 * hc + 16 * jj;  // TMEM column of the chunk within S^T / dP^T
          tmem_ld16x2(tS + col + lane_off, sv, tdP + col + lane_off, pv);
          if (jj == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_st_free[b]);
          }
          const int col0 = 64 * b + 32 * hc + 16 * jj;  // query column within the 128-query tile
          const float* st = sStat + hs * 64 + 32 * hc + 16 * jj;
          const float* dd = sDi + hs * 64 + 32 * hc + 16 * jj;
          if (ii == 0)
            grads_chunk<N, CLIP, INV_STAT, true, 16, SHIFTED>(sv, pv, st, dd, pk[jj], dk2[jj], cfg.clamp, col0, r);
          else
            grads_chunk<N, CLIP, INV_STAT, false, 16, SHIFTED>(sv, pv, st, dd, pk[jj], dk2[jj], cfg.clamp, col0, r);
        }
        // P^T of sub-tile Ug - 2 must have been consumed by its dV product,
        // dS^T of query tile Ig - 2 by its dQ product.
        if (Ug >= 2 && !mbar_wait_warp(&bar_p_free[b], ((Ug >> 1) - 1) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
        // bf16 P^T pairs of this warp's 32 query columns -> 16 TMEM columns of
        // P^T[b]; the store completes while dS^T goes to shared memory.
        uint32_t pv16[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pv16[i] = pk[0][i];
          pv16[8 + i] = pk[1][i];
        }
        tmem_st16_nowait(tPT + 32 * b + 16 * hc + lane_off, pv16);
        const int c16 = 8 * b + 4 * hc;  // first 16-byte unit of this warp's 32 columns
        if (Ig >= 2 && !mbar_wait_warp(&bar_ds_free[s], ((Ig >> 1) - 1) & 1, abort_v, dev_err)) {
          tmem_wait_st(pv16);
          ok = false;
          break;
        }
        uint8_t* ds_tile = sdST + s * 2 * kTileBytes;
#pragma unroll
        for (int un = 0; un < 4; ++un) {
          const uint32_t* v = dk2[un >> 1] + 4 * (un & 1);
          *reinterpret_cast<uint4*>(ds_tile + sw128_off(r, c16 + un)) = make_uint4(v[0], v[1], v[2], v[3]);
        }
        tmem_wait_st(pv16);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bar_ps_ready[b]);
          mbar_arrive(&bar_ds_ready[s]);
        }
      }
      U += nu;
      I += w.ni;
    }
  } else if (warp < kBwdDrain + 4) {
    // ----- dQ drain and the items' dK / dV write-out: thread owns TMEM lane r.
    // dQ goes out in two rounds per tile (columns 0-31, then 32-63) through
    // two alternating 16 KB staging boxes, so the stores of one round overlap
    // the reduce-add of the previous; row r, 16-byte chunk c of a 128-byte box
    // row sits at chunk c ^ (r & 7). The write-out of an item comes before the
    // drain of its last dQ tile: the next item's first dV / dK products wait
    // for it.
    const int dw = warp - kBwdDrain, r = dw * 32 + lane;
    const uint32_t lane_off = (uint32_t)(dw * 32) << 16;
    const bool issuer = dw == 0 && lane == 0;
    int I = 0, rounds = 0;
    bool ok = true;
    // drain dQ tile I (query rows y..y+127) through the box
    auto drain_tile = [&](int y) -> bool {
      if (!mbar_wait_warp(&bar_dq_full, I & 1, abort_v, dev_err)) return false;
      for (int h = 0; h < 2; ++h, ++rounds) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tdQ + 32 * h + lane_off, v);
        if (h == 1) {  // both halves read: the next tile's product may overwrite TMEM
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar_dq_free);
        }
        const int sb = rounds & 1;
        uint8_t* box = sDQ + sb * kTileBytes;
        if (rounds >= 2 && !mbar_wait_warp(&bar_stage_free[sb], ((rounds >> 1) - 1) & 1, abort_v, dev_err))
          return false;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(box + r * 128 + ((c ^ (r & 7)) << 4)) =
              make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_stage_full[sb]);
        bool good = true;
        if (issuer) {
          if (mbar_wait(&bar_stage_full[sb], (rounds >> 1) & 1, abort_v, dev_err)) {
            tma_reduce_add_2d(&tdq, box, 32 * h, y);
            bulk_commit_group();
            if (rounds >= 1) {  // the previous round's box has been read: release it
              bulk_wait_group_read1();
              mbar_arrive(&bar_stage_free[sb ^ 1]);
            }
          } else {
            good = false;
          }
        }
        __syncwarp();
        if (!__all_sync(0xffffffffu, good)) return false;
      }
      ++I;
      return true;
    };
    for (int j = 0; ok; ++j) {
      const int it = next_item(j, true);
      if (it < 0) break;
      const BwdItem w = bwd_item(it, BH, nq);
      const int row_base = w.bh * T;
      for (int ii = 0; ok && ii + 1 < w.ni; ++ii) ok = drain_tile(row_base + (w.kt + ii) * kTile);
      // dK = n * acc and dV = acc, rounded to bf16, leave through the staging
      // boxes as two swizzled 128 x 64 tiles with TMA stores; TMEM is free for
      // the next item as soon as both accumulators are in registers.
      if (!ok || !mbar_wait_warp(&bar_fin, j & 1, abort_v, dev_err)) {
        ok = false;
        break;
      }
      const int key_row = row_base + w.kt * kTile;
      for (int which = 0; ok && which < 2; ++which, ++rounds) {
        const int sb = rounds & 1;
        uint8_t* box = sDQ + sb * kTileBytes;
        if (rounds >= 2 && !mbar_wait_warp(&bar_stage_free[sb], ((rounds >> 1) - 1) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
        const float f = which == 0 ? (float)N : 1.f;
#pragma unroll 1
        for (int part = 0; part < 2; ++part) {
          tc_fence_after();
          uint32_t v[32];
          tmem_ld32((which == 0 ? tdK : tdV) + lane_off + 32 * part, v);
          if (which == 1 && part == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_acc_free);
          }
#pragma unroll
          for (int un = 0; un < 4; ++un) {
            uint4 q;
            q.x = pack_bf16x2(__uint_as_float(v[8 * un + 0]) * f, __uint_as_float(v[8 * un + 1]) * f);
            q.y = pack_bf16x2(__uint_as_float(v[8 * un + 2]) * f, __uint_as_float(v[8 * un + 3]) * f);
            q.z = pack_bf16x2(__uint_as_float(v[8 * un + 4]) * f, __uint_as_float(v[8 * un + 5]) * f);
            q.w = pack_bf16x2(__uint_as_float(v[8 * un + 6]) * f, __uint_as_float(v[8 * un + 7]) * f);
            const int c = 4 * part + un;  // 16-byte unit (8 columns) of the 128-byte row
            *reinterpret_cast<uint4*>(box + r * 128 + ((c ^ (r & 7)) << 4)) = q;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_stage_full[sb]);
        bool good = true;
        if (issuer) {
          if (mbar_wait(&bar_stage_full[sb], (rounds >> 1) & 1, abort_v, dev_err)) {
            tma_store_2d(which == 0 ? &tdk : &tdv, box, 0, key_row);
            bulk_commit_group();
            if (rounds >= 1) {
              bulk_wait_group_read1();
              mbar_arrive(&bar_stage_free[sb ^ 1]);
            }
          } else {
            good = false;
          }
        }
        __syncwarp();
        if (!__all_sync(0xffffffffu, good)) ok = false;
      }
      if (!ok) break;
      ok = drain_tile(row_base + (w.kt + w.ni - 1) * kTile);
    }
    if (issuer) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kBwdProducer) tmem_dealloc(tmem_base, 512);
}

// dq = bf16(acc * n * scale), for the branch a tcgen05 backward ran: the
// unshifted one, and with the range guard the shifted one as well.
__global__ void dq_finish_kernel(algx_attn_config cfg, const float* __restrict__ guard,
                                 const float4* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t n4) {
  pdl_wait();  // launched as a dependent of the fast backward
  pdl_trigger();  // the fallback kernels may be scheduled behind this grid
  const Eff e = resolve_variant(cfg, guard);
  if (!tc_bwd_covers(cfg, e)) return;
  const float f = (float)cfg.n * cfg.scale;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = acc[i];
    uint2 w;
    w.x = pack_bf16x2(a.x * f, a.y * f);
    w.y = pack_bf16x2(a.z * f, a.w * f);
    reinterpret_cast<uint2*>(dq)[i] = w;
  }
}

bool fast_eligible(const algx_attn_config& cfg, int64_t T, int32_t dtype) {
  if (dtype != ALGX_BF16 || T % kTile != 0 || T < kTile) return false;
  if (cfg.kind != ALGX_ATTN_ASINH || !cfg.fast_rho) return false;
  if (cfg.mode != ALGX_MODE_CLIPPED && cfg.mode != ALGX_MODE_GUARDED) return false;
  if (cfg.n != 8 && cfg.n != 16 && cfg.n != 32) return false;
  // guarded low branch always uses the 1/Z statistic
  return true;
}

template <int N, bool CLIP>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const algx_attn_config& cfg,
               const float* sink, const float* guard, void* o, float* o_prec, float* stat, int64_t B, int64_t H,
               int64_t T, cudaStream_t st) {
  auto kern = attn_fwd_tc_kernel<N, CLIP>;
  ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
  dim3 grid((unsigned)(B * H), (unsigned)(T / kTile));
  ALGX_CUDA(launch_dependent(kern, grid, kFwdThreads, kFwdSmem, st, tq, tk, tv, cfg, sink, guard,
                             static_cast<__nv_bfloat16*>(o), o_prec, stat, (int)H, (int)T, device_error_word()));
  ALGX_LAUNCHED("attn_fwd_tc launch");
  return ALGX_OK;
}

template <int N, bool CLIP, bool INV, bool SHIFTED = false>
int launch_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
               const CUtensorMap& tdq, const CUtensorMap& tdk, const CUtensorMap& tdv, const algx_attn_config& cfg,
               const float* stat, const float* di, const float* guard, int* item_counter, int64_t B, int64_t H,
               int64_t T, cudaStream_t st) {
  auto kern = attn_bwd_tc_kernel<N, CLIP, INV, SHIFTED>;
  ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem));
  int dev = 0, sms = 0;
  ALGX_CUDA(cudaGetDevice(&dev));
  ALGX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t items = B * H * (T / kTile);
  const unsigned grid = (unsigned)std::min<int64_t>(items, sms);  // persistent: one CTA per SM
  ALGX_CUDA(launch_dependent(kern, grid, kBwdThreads, kBwdSmem, st, tq, tk, tv, tdo, tdq, tdk, tdv, cfg, stat, di,
                             guard, item_counter, (int)(B * H), (int)T, device_error_word()));
  ALGX_LAUNCHED("attn_bwd_tc launch");
  return ALGX_OK;
}

int make_maps(const void* const* ptrs, int count, CUtensorMap* maps, int64_t rows) {
  for (int i = 0; i < count; ++i)
    if (int s = make_tmap_2d(&maps[i], ptrs[i], ALGX_BF16, 64, (uint64_t)rows, 128, 64, kTile, true)) return s;
  return ALGX_OK;
}

}  // namespace

int tc_attn_fwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v, const float* sink,
                const float* guard, void* o, float* o_prec, float* stat, int64_t B, int64_t H, int64_t T,
                int32_t dtype, cudaStream_t st, bool* launched) {
  *launched = false;
  if (!fast_eligible(cfg, T, dtype)) return ALGX_OK;
  CUtensorMap maps[3];
  const void* ptrs[3] = {q_scaled, k, v};
  if (int s = make_maps(ptrs, 3, maps, B * H * T)) return s;
  const bool clip = cfg.mode == ALGX_MODE_CLIPPED;
  int s;
  if (cfg.n == 16)
    s = clip ? launch_fwd<16, true>(maps[0], maps[1], maps[2], cfg, sink, guard, o, o_prec, stat, B, H, T, st)
             : launch_fwd<16, false>(maps[0], maps[1], maps[2], cfg, sink, guard, o, o_prec, stat, B, H, T, st);
  else if (cfg.n == 8)
    s = clip ? launch_fwd<8, true>(maps[0], maps[1], maps[2], cfg, sink, guard, o, o_prec, stat, B, H, T, st)
             : launch_fwd<8, false>(maps[0], maps[1], maps[2], cfg, sink, guard, o, o_prec, stat, B, H, T, st);
  else
    s = clip ? launch_fwd<32, true>(maps[0], maps[1], maps[2], cfg, sink, guard, o, o_prec, stat, B, H, T, st)
             : launch_fwd<32, false>(maps[0], maps[1], maps[2], cfg, sink, guard, o, o_prec, stat, B, H, T, st);
  if (s) return s;
  *launched = true;
  return ALGX_OK;
}

// fp32 dQ accumulator, then the persistent kernel's work-item counter and
// spare bytes for the caller (all zeroed by one memset per call).
size_t tc_attn_bwd_workspace(int64_t B, int64_t H, int64_t T, int64_t D) {
  return (size_t)B * H * T * D * sizeof(float) + 256;
}
bool tc_attn_bwd_eligible(const algx_attn_config& cfg, int64_t T, int32_t dtype) {
  return fast_eligible(cfg, T, dtype);
}
size_t tc_attn_bwd_spare_offset(int64_t B, int64_t H, int64_t T, int64_t D) {
  return (size_t)B * H * T * D * sizeof(float) + 128;
}

int tc_attn_bwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v, const void* dout,
                const float* stat, const float* di, const float* guard, void* dq, void* dk, void* dv, void* workspace,
                int64_t B, int64_t H, int64_t T, int32_t dtype, cudaStream_t st, bool finish_dq, bool pre_zeroed,
                bool* launched) {
  *launched = false;
  if (!fast_eligible(cfg, T, dtype)) return ALGX_OK;
  CUtensorMap maps[6];  // q, k, v, dO (loads), dK, dV (stores)
  const void* ptrs[6] = {q_scaled, k, v, dout, dk, dv};
  if (int s = make_maps(ptrs, 6, maps, B * H * T)) return s;
  // Q and dO stream in 64-query halves
  for (int i : {0, 3})
    if (int s = make_tmap_2d(&maps[i], ptrs[i], ALGX_BF16, 64, (uint64_t)(B * H * T), 128, 64, 64, true)) return s;
  float* acc = static_cast<float*>(workspace);
  const size_t nacc = (size_t)B * H * T * 64;
  CUtensorMap tdq;  // fp32 accumulator, reduce-added in 128-row x 32-column boxes
  if (int s = make_tmap_2d(&tdq, acc, ALGX_F32, 64, (uint64_t)(B * H * T), 256, 32, kTile, true)) return s;
  int* item_counter = reinterpret_cast<int*>(acc + nacc);
  if (!pre_zeroed) ALGX_CUDA(cudaMemsetAsync(acc, 0, nacc * sizeof(float) + 256, st));
  const bool clip = cfg.mode == ALGX_MODE_CLIPPED;
  // The guarded low branch uses the 1/Z statistic; the clipped link follows cfg.inv_stat.
  const bool inv = clip ? cfg.inv_stat != 0 : true;
  int s;
#define ALGX_BWD(NN, CC, II, SS) \
  launch_bwd<NN, CC, II, SS>(maps[0], maps[1], maps[2], maps[3], tdq, maps[4], maps[5], cfg, stat, di, guard, \
                             item_counter, B, H, T, st)
  if (cfg.n == 16)
    s = clip ? (inv ? ALGX_BWD(16, true, true, false) : ALGX_BWD(16, true, false, false))
             : ALGX_BWD(16, false, true, false);
  else if (cfg.n == 8)
    s = clip ? (inv ? ALGX_BWD(8, true, true, false) : ALGX_BWD(8, true, false, false))
             : ALGX_BWD(8, false, true, false);
  else
    s = clip ? (inv ? ALGX_BWD(32, true, true, false) : ALGX_BWD(32, true, false, false))
             : ALGX_BWD(32, false, true, false);
  if (s) return s;
  // With the range guard, the shifted branch's backward on the same pipeline
  // (it returns at once unless the guard chose that branch).
  if (cfg.mode == ALGX_MODE_GUARDED) {
    s = cfg.n == 16 ? ALGX_BWD(16, false, false, true)
                    : (cfg.n == 8 ? ALGX_BWD(8, false, false, true) : ALGX_BWD(32, false, false, true));
    if (s) return s;
  }
#undef ALGX_BWD
  if (finish_dq) {
    const int64_t n4 = (int64_t)(nacc / 4);
    const int grid = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 16);
    ALGX_CUDA(launch_dependent(dq_finish_kernel, grid, 256, 0, st, cfg, guard, reinterpret_cast<const float4*>(acc),
                               static_cast<__nv_bfloat16*>(dq), n4));
    ALGX_LAUNCHED("dq_finish launch");
  }
  *launched = true;
  return ALGX_OK;
}

}  // namespace algx
