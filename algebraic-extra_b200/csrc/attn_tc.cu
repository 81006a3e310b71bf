// tcgen05 attention fast path: bf16 I/O, D = 64, T % 128 == 0, asinh
// unshifted branch (the guarded low branch or the explicit clipped link),
// fast rho, n in {8, 16, 32}.
//
// Forward (kernels/flash.py:189-284, head_resident.py:24-93): one CTA per
// (128-query tile, head), two CTAs per SM. Warp roles: warps 0-3 compute the
// weights (thread = query row = TMEM lane), warp 4 issues TMA loads, warp 5
// issues tcgen05 MMAs. S = Q K^T lands in TMEM (fp32), the weight warps turn
// each row into p = rho(x)^n, accumulate the fp32 row sum, and write bf16 P
// back into TMEM; O += P V reads P from TMEM (A operand) and V from shared
// memory (MN-major). No running maximum exists on this branch, so O needs no
// rescaling; O = acc / l and stat = 1/l (or l^(-1/n)) at the end.
//
// Backward (kernels/flash.py:333-361, 435-627): one CTA per (128-key tile,
// head). K, V stay resident; query tiles stream through a 2-stage TMA ring.
// Per query tile: S^T = K Q^T and dP^T = V dO^T in TMEM; warps 0-3 (thread =
// key row) recompute p = rho^n * stat, ds = p (dp - di) r, write bf16 P^T and
// dS^T to shared memory (128-byte swizzled K-major); then dV += P^T dO,
// dK += dS^T Q, and dQ_tile = dS K (the same dS^T buffer read MN-major).
// Warps 4-7 drain dQ_tile from TMEM into an fp32 accumulator with vector
// reductions; a final pass scales and rounds it. Every mbarrier wait is
// bounded (sm100.cuh).
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
constexpr int kFwdStages = 2;
constexpr int kFwdThreads = 192;
constexpr int kFwdSmem = kTileBytes * (1 + 2 * kFwdStages) + 1024;
constexpr int kBwdThreads = 320;
constexpr int kBwdSmem = kTileBytes * 10 + 4 * kTile * 4 + 1024;

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

// ---------------------------------------------------------------- forward
template <int N, bool CLIP>
__global__ void __launch_bounds__(kFwdThreads, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, algx_attn_config cfg, const float* __restrict__ sink,
                       const float* __restrict__ guard, __nv_bfloat16* __restrict__ o, float* __restrict__ stat,
                       int H, int T, int* dev_err) {
  const Eff e = resolve_variant(cfg, guard);
  if (e.branch != BR_UNSHIFTED) return;  // the generic kernel runs the shifted fallback
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kTileBytes;
  uint8_t* sV = sK + kFwdStages * kTileBytes;
  __shared__ uint64_t bar_q, bar_s_full, bar_p_full, bar_p_free, bar_o_full;
  __shared__ uint64_t bar_kv_full[kFwdStages], bar_kv_empty[kFwdStages];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = T / kTile;
  const int qt = nq - 1 - (int)blockIdx.x;  // longest rows first
  const int bh = blockIdx.y;
  const int nk = qt + 1;
  const int row_base = bh * T;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    mbar_init(&bar_s_full, 1);
    mbar_init(&bar_p_full, 4);
    mbar_init(&bar_p_free, 1);
    mbar_init(&bar_o_full, 1);
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&bar_kv_full[s], 1);
      mbar_init(&bar_kv_empty[s], 1);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 4) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = tmem_base, tO = tmem_base + 128, tP = tmem_base + 192;

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      mbar_expect_tx(&bar_q, kTileBytes);
      tma_load_2d(sQ, &tq, &bar_q, 0, row_base + qt * kTile);
      int issued[kFwdStages] = {-1, -1};
      for (int j = 0; j < nk; ++j) {
        const int s = j % kFwdStages;
        if (j >= kFwdStages && !mbar_wait(&bar_kv_empty[s], ((j / kFwdStages) - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&bar_kv_full[s], 2 * kTileBytes);
        tma_load_2d(sK + s * kTileBytes, &tk, &bar_kv_full[s], 0, row_base + j * kTile);
        tma_load_2d(sV + s * kTileBytes, &tv, &bar_kv_full[s], 0, row_base + j * kTile);
        issued[s] = j;
      }
      if (*abort_v) {  // let copies in flight land before the CTA exits
        for (int s = 0; s < kFwdStages; ++s)
          if (issued[s] >= 0) {
            volatile int quiet = 0;
            mbar_wait(&bar_kv_full[s], (issued[s] / kFwdStages) & 1, &quiet, nullptr);
          }
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t idS = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idO = idesc_bf16_f32(128, 64, 0, 1);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK), v0 = smem_u32(sV);
      bool ok = mbar_wait(&bar_q, 0, abort_v, dev_err);
      for (int j = 0; ok && j < nk; ++j) {
        const int s = j % kFwdStages;
        if (!mbar_wait(&bar_kv_full[s], (j / kFwdStages) & 1, abort_v, dev_err)) break;
        if (j > 0 && !mbar_wait(&bar_p_full, (j - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t kb = k0 + s * kTileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_ss(tS, desc_sw128(q0 + k * 32, 16, 1024), desc_sw128(kb + k * 32, 16, 1024), idS, k > 0);
        mma_commit(&bar_s_full);
        if (j > 0) {
          const int sp = (j - 1) % kFwdStages;
          const uint32_t vb = v0 + sp * kTileBytes;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_ts(tO, tP + k * 8, desc_sw128(vb + k * 2048, 8192, 1024), idO, (j - 1 > 0 || k > 0));
          mma_commit(&bar_p_free);
          mma_commit(&bar_kv_empty[sp]);
        }
      }
      if (!*abort_v && mbar_wait(&bar_p_full, (nk - 1) & 1, abort_v, dev_err)) {
        tc_fence_after();
        const int sp = (nk - 1) % kFwdStages;
        const uint32_t vb = v0 + sp * kTileBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_ts(tO, tP + k * 8, desc_sw128(vb + k * 2048, 8192, 1024), idO, (nk - 1 > 0 || k > 0));
        mma_commit(&bar_o_full);
      }
    }
  } else {
    // ----- weight warps: thread r owns query row qt*128 + r (TMEM lane r)
    const int r = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float l = 0.f, rr;
    if (cfg.has_sink) l = weight<N, CLIP>(sink[bh % H], cfg.clamp, rr);
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      if (!mbar_wait_warp(&bar_s_full, j & 1, abort_v, dev_err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = j == qt;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32];
        tmem_ld32(tS + lane_off + c * 32, sv);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float p0 = weight<N, CLIP>(__uint_as_float(sv[2 * i]), cfg.clamp, rr);
          float p1 = weight<N, CLIP>(__uint_as_float(sv[2 * i + 1]), cfg.clamp, rr);
          if (diag) {
            const int col = c * 32 + 2 * i;
            if (col > r) p0 = 0.f;
            if (col + 1 > r) p1 = 0.f;
          }
          l += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        if (c == 0 && j > 0 && !mbar_wait_warp(&bar_p_free, (j - 1) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
        tmem_st16(tP + lane_off + c * 16, pk);
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p_full);
    }
    if (ok && mbar_wait_warp(&bar_o_full, 0, abort_v, dev_err)) {
      tc_fence_after();
      const float inv = 1.f / l;
      const size_t row = (size_t)row_base + (size_t)qt * kTile + r;
      uint4* dst = reinterpret_cast<uint4*>(o + row * 64);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t ov[32];
        tmem_ld32(tO + lane_off + c * 32, ov);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(ov[8 * u + 0]) * inv, __uint_as_float(ov[8 * u + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(ov[8 * u + 2]) * inv, __uint_as_float(ov[8 * u + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(ov[8 * u + 4]) * inv, __uint_as_float(ov[8 * u + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(ov[8 * u + 6]) * inv, __uint_as_float(ov[8 * u + 7]) * inv);
          dst[c * 4 + u] = w;
        }
      }
      stat[row] = e.inv_stat ? inv : inv_root(l, N);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem_base, 256);
}

// ---------------------------------------------------------------- backward
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Byte offset of bf16 element (row, col) in a [128 rows][128 cols] tile kept
// as two 128-byte-swizzled K-major halves of 64 columns.
__device__ __forceinline__ uint32_t sw128_off(int row, int col16) {
  // col16: index of the 16-byte unit (8 bf16) in [0, 16)
  const int half = col16 >> 3, u = col16 & 7;
  return half * kTileBytes + row * 128 + ((u ^ (row & 7)) << 4);
}

template <int N, bool CLIP, bool INV_STAT>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                       const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                       algx_attn_config cfg, const float* __restrict__ stat, const float* __restrict__ di,
                       const float* __restrict__ guard, float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dk,
                       __nv_bfloat16* __restrict__ dv, int T, int* dev_err) {
  const Eff e = resolve_variant(cfg, guard);
  if (e.branch != BR_UNSHIFTED) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTileBytes;
  uint8_t* sQ = smem + 2 * kTileBytes;    // 2 stages
  uint8_t* sdO = smem + 4 * kTileBytes;   // 2 stages
  uint8_t* sPT = smem + 6 * kTileBytes;   // 128 keys x 128 queries bf16 (2 halves)
  uint8_t* sdST = smem + 8 * kTileBytes;  // idem
  float* sStat = reinterpret_cast<float*>(smem + 10 * kTileBytes);  // [2][128]
  float* sDi = sStat + 2 * kTile;                                    // [2][128]
  __shared__ uint64_t bar_kv, bar_st_full, bar_ps_ready, bar_ps_free, bar_dq_full, bar_dq_free, bar_fin;
  __shared__ uint64_t bar_qd_full[2], bar_qd_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = T / kTile;
  const int kt = (int)blockIdx.x;  // key tile; kt = 0 has the most query tiles
  const int bh = blockIdx.y;
  const int row_base = bh * T;
  const int ni = nq - kt;  // query tiles kt .. nq-1

  if (threadIdx.x == 0) {
    mbar_init(&bar_kv, 1);
    mbar_init(&bar_st_full, 1);
    mbar_init(&bar_ps_ready, 4);
    mbar_init(&bar_ps_free, 1);
    mbar_init(&bar_dq_full, 1);
    mbar_init(&bar_dq_free, 4);
    mbar_init(&bar_fin, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_qd_full[s], 1);
      mbar_init(&bar_qd_empty[s], 1);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 8) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = tmem_base, tdP = tmem_base + 128, tdV = tmem_base + 256, tdK = tmem_base + 320,
                 tdQ = tmem_base + 384;

  if (warp == 8) {
    // ----- producer
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&tdo);
      mbar_expect_tx(&bar_kv, 2 * kTileBytes);
      tma_load_2d(sK, &tk, &bar_kv, 0, row_base + kt * kTile);
      tma_load_2d(sV, &tv, &bar_kv, 0, row_base + kt * kTile);
      int issued[2] = {-1, -1};
      for (int ii = 0; ii < ni; ++ii) {
        const int s = ii & 1, qi = kt + ii;
        if (ii >= 2 && !mbar_wait(&bar_qd_empty[s], ((ii >> 1) - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&bar_qd_full[s], 2 * kTileBytes + 2 * kTile * 4);
        tma_load_2d(sQ + s * kTileBytes, &tq, &bar_qd_full[s], 0, row_base + qi * kTile);
        tma_load_2d(sdO + s * kTileBytes, &tdo, &bar_qd_full[s], 0, row_base + qi * kTile);
        bulk_load(sStat + s * kTile, stat + row_base + qi * kTile, kTile * 4, &bar_qd_full[s]);
        bulk_load(sDi + s * kTile, di + row_base + qi * kTile, kTile * 4, &bar_qd_full[s]);
        issued[s] = ii;
      }
      if (*abort_v) {
        for (int s = 0; s < 2; ++s)
          if (issued[s] >= 0) {
            volatile int quiet = 0;
            mbar_wait(&bar_qd_full[s], (issued[s] >> 1) & 1, &quiet, nullptr);
          }
      }
    }
  } else if (warp == 9) {
    // ----- MMA issuer
    if (lane == 0) {
      const uint32_t idS = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t idKM = idesc_bf16_f32(128, 64, 0, 1);  // A K-major smem, B MN-major
      const uint32_t idMM = idesc_bf16_f32(128, 64, 1, 1);  // A MN-major smem, B MN-major
      const uint32_t k0 = smem_u32(sK), v0 = smem_u32(sV), q0 = smem_u32(sQ), do0 = smem_u32(sdO);
      const uint32_t pt0 = smem_u32(sPT), ds0 = smem_u32(sdST);
      bool ok = mbar_wait(&bar_kv, 0, abort_v, dev_err);
      auto consume = [&](int ii) -> bool {  // dV, dK, dQ of query tile ii
        const int s = ii & 1;
        const uint32_t qb = q0 + s * kTileBytes, db = do0 + s * kTileBytes;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_ss(tdV, desc_sw128(pt0 + (k >> 2) * kTileBytes + (k & 3) * 32, 16, 1024),
                 desc_sw128(db + k * 2048, 8192, 1024), idKM, (ii > 0 || k > 0));
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_ss(tdK, desc_sw128(ds0 + (k >> 2) * kTileBytes + (k & 3) * 32, 16, 1024),
                 desc_sw128(qb + k * 2048, 8192, 1024), idKM, (ii > 0 || k > 0));
        mma_commit(&bar_qd_empty[s]);
        if (ii > 0 && !mbar_wait(&bar_dq_free, (ii - 1) & 1, abort_v, dev_err)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_ss(tdQ, desc_sw128(ds0 + k * 2048, kTileBytes, 1024), desc_sw128(k0 + k * 2048, 8192, 1024), idMM,
                 k > 0);
        mma_commit(&bar_dq_full);
        mma_commit(&bar_ps_free);
        return true;
      };
      for (int ii = 0; ok && ii < ni; ++ii) {
        const int s = ii & 1;
        if (!mbar_wait(&bar_qd_full[s], (ii >> 1) & 1, abort_v, dev_err)) break;
        if (ii > 0 && !mbar_wait(&bar_ps_ready, (ii - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t qb = q0 + s * kTileBytes, db = do0 + s * kTileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_ss(tS, desc_sw128(k0 + k * 32, 16, 1024), desc_sw128(qb + k * 32, 16, 1024), idS, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_ss(tdP, desc_sw128(v0 + k * 32, 16, 1024), desc_sw128(db + k * 32, 16, 1024), idS, k > 0);
        mma_commit(&bar_st_full);
        if (ii > 0 && !consume(ii - 1)) break;
      }
      if (!*abort_v && mbar_wait(&bar_ps_ready, (ni - 1) & 1, abort_v, dev_err) && consume(ni - 1))
        mma_commit(&bar_fin);
    }
  } else if (warp < 4) {
    // ----- score-gradient warps: thread r owns key row kt*128 + r (TMEM lane r)
    const int r = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    bool ok = true;
    for (int ii = 0; ii < ni; ++ii) {
      const int s = ii & 1;
      if (!mbar_wait_warp(&bar_st_full, ii & 1, abort_v, dev_err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = ii == 0;  // query tile == key tile
      const float* st = sStat + s * kTile;
      const float* dd = sDi + s * kTile;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32], pv[32];
        tmem_ld32(tS + lane_off + c * 32, sv);
        tmem_ld32(tdP + lane_off + c * 32, pv);
        uint32_t pk[16], dk2[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float pp[2], dd2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int col = c * 32 + 2 * i + h;
            const float sc = __uint_as_float(sv[2 * i + h]);
            const float x = CLIP ? fminf(sc, cfg.clamp) : sc;
            const float rad = fmaf(x, x, 1.f);
            const float rr = rsqrtf(rad);
            const float rho = fmaf(rad, rr, x);
            const float stc = st[col];
            float p = INV_STAT ? ipow_t<N>(rho) * stc : ipow_t<N>(rho * stc);
            float ds = p * (__uint_as_float(pv[2 * i + h]) - dd[col]) * rr;
            if constexpr (CLIP) ds = sc < cfg.clamp ? ds : 0.f;
            if (diag && col < r) {
              p = 0.f;
              ds = 0.f;
            }
            pp[h] = p;
            dd2[h] = ds;
          }
          pk[i] = pack_bf16x2(pp[0], pp[1]);
          dk2[i] = pack_bf16x2(dd2[0], dd2[1]);
        }
        if (c == 0 && ii > 0 && !mbar_wait_warp(&bar_ps_free, (ii - 1) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t off = sw128_off(r, c * 4 + u);
          *reinterpret_cast<uint4*>(sPT + off) = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
          *reinterpret_cast<uint4*>(sdST + off) =
              make_uint4(dk2[4 * u], dk2[4 * u + 1], dk2[4 * u + 2], dk2[4 * u + 3]);
        }
      }
      if (!ok) break;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_ps_ready);
    }
    if (ok && mbar_wait_warp(&bar_fin, 0, abort_v, dev_err)) {
      tc_fence_after();
      const size_t row = (size_t)row_base + (size_t)kt * kTile + r;
      const float slope = (float)N;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        __nv_bfloat16* dst = which == 0 ? dk : dv;
        const uint32_t tsrc = which == 0 ? tdK : tdV;
        const float f = which == 0 ? slope : 1.f;
        uint4* d4 = reinterpret_cast<uint4*>(dst + row * 64);
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld32(tsrc + lane_off + c * 32, v);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * u + 0]) * f, __uint_as_float(v[8 * u + 1]) * f);
            w.y = pack_bf16x2(__uint_as_float(v[8 * u + 2]) * f, __uint_as_float(v[8 * u + 3]) * f);
            w.z = pack_bf16x2(__uint_as_float(v[8 * u + 4]) * f, __uint_as_float(v[8 * u + 5]) * f);
            w.w = pack_bf16x2(__uint_as_float(v[8 * u + 6]) * f, __uint_as_float(v[8 * u + 7]) * f);
            d4[c * 4 + u] = w;
          }
        }
      }
    }
  } else {
    // ----- dQ drain warps 4-7: thread owns query row qi*128 + (threadIdx.x - 128) (TMEM lane)
    const int r = threadIdx.x - 128;
    const uint32_t lane_off = (uint32_t)((warp - 4) * 32) << 16;
    for (int ii = 0; ii < ni; ++ii) {
      if (!mbar_wait_warp(&bar_dq_full, ii & 1, abort_v, dev_err)) break;
      tc_fence_after();
      uint32_t a[32], b[32];
      tmem_ld32(tdQ + lane_off, a);
      tmem_ld32(tdQ + lane_off + 32, b);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_dq_free);
      float* dst = dq_acc + ((size_t)row_base + (size_t)(kt + ii) * kTile + r) * 64;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        red_add_v4(dst + 4 * u, __uint_as_float(a[4 * u]), __uint_as_float(a[4 * u + 1]),
                   __uint_as_float(a[4 * u + 2]), __uint_as_float(a[4 * u + 3]));
#pragma unroll
      for (int u = 0; u < 8; ++u)
        red_add_v4(dst + 32 + 4 * u, __uint_as_float(b[4 * u]), __uint_as_float(b[4 * u + 1]),
                   __uint_as_float(b[4 * u + 2]), __uint_as_float(b[4 * u + 3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) tmem_dealloc(tmem_base, 512);
}

// dq = bf16(acc * n * scale), only when the fast path ran (unshifted branch).
__global__ void dq_finish_kernel(algx_attn_config cfg, const float* __restrict__ guard,
                                 const float4* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t n4) {
  const Eff e = resolve_variant(cfg, guard);
  if (e.branch != BR_UNSHIFTED) return;
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
               const float* sink, const float* guard, void* o, float* stat, int64_t B, int64_t H, int64_t T,
               cudaStream_t st) {
  auto kern = attn_fwd_tc_kernel<N, CLIP>;
  ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
  dim3 grid((unsigned)(T / kTile), (unsigned)(B * H));
  kern<<<grid, kFwdThreads, kFwdSmem, st>>>(tq, tk, tv, cfg, sink, guard, static_cast<__nv_bfloat16*>(o), stat,
                                            (int)H, (int)T, device_error_word());
  ALGX_LAUNCHED("attn_fwd_tc launch");
  return ALGX_OK;
}

template <int N, bool CLIP, bool INV>
int launch_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
               const algx_attn_config& cfg, const float* stat, const float* di, const float* guard, float* dq_acc,
               void* dk, void* dv, int64_t B, int64_t H, int64_t T, cudaStream_t st) {
  auto kern = attn_bwd_tc_kernel<N, CLIP, INV>;
  ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem));
  dim3 grid((unsigned)(T / kTile), (unsigned)(B * H));
  kern<<<grid, kBwdThreads, kBwdSmem, st>>>(tq, tk, tv, tdo, cfg, stat, di, guard, dq_acc,
                                            static_cast<__nv_bfloat16*>(dk), static_cast<__nv_bfloat16*>(dv),
                                            (int)T, device_error_word());
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
                const float* guard, void* o, float* stat, int64_t B, int64_t H, int64_t T, int32_t dtype,
                cudaStream_t st, bool* launched) {
  *launched = false;
  if (!fast_eligible(cfg, T, dtype)) return ALGX_OK;
  CUtensorMap maps[3];
  const void* ptrs[3] = {q_scaled, k, v};
  if (int s = make_maps(ptrs, 3, maps, B * H * T)) return s;
  const bool clip = cfg.mode == ALGX_MODE_CLIPPED;
  int s;
  if (cfg.n == 16)
    s = clip ? launch_fwd<16, true>(maps[0], maps[1], maps[2], cfg, sink, guard, o, stat, B, H, T, st)
             : launch_fwd<16, false>(maps[0], maps[1], maps[2], cfg, sink, guard, o, stat, B, H, T, st);
  else if (cfg.n == 8)
    s = clip ? launch_fwd<8, true>(maps[0], maps[1], maps[2], cfg, sink, guard, o, stat, B, H, T, st)
             : launch_fwd<8, false>(maps[0], maps[1], maps[2], cfg, sink, guard, o, stat, B, H, T, st);
  else
    s = clip ? launch_fwd<32, true>(maps[0], maps[1], maps[2], cfg, sink, guard, o, stat, B, H, T, st)
             : launch_fwd<32, false>(maps[0], maps[1], maps[2], cfg, sink, guard, o, stat, B, H, T, st);
  if (s) return s;
  *launched = true;
  return ALGX_OK;
}

size_t tc_attn_bwd_workspace(int64_t B, int64_t H, int64_t T, int64_t D) {
  return (size_t)B * H * T * D * sizeof(float);
}

int tc_attn_bwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v, const void* dout,
                const float* stat, const float* di, const float* guard, void* dq, void* dk, void* dv, void* workspace,
                int64_t B, int64_t H, int64_t T, int32_t dtype, cudaStream_t st, bool* launched) {
  *launched = false;
  if (!fast_eligible(cfg, T, dtype)) return ALGX_OK;
  CUtensorMap maps[4];
  const void* ptrs[4] = {q_scaled, k, v, dout};
  if (int s = make_maps(ptrs, 4, maps, B * H * T)) return s;
  float* acc = static_cast<float*>(workspace);
  const size_t nacc = (size_t)B * H * T * 64;
  ALGX_CUDA(cudaMemsetAsync(acc, 0, nacc * sizeof(float), st));
  const bool clip = cfg.mode == ALGX_MODE_CLIPPED;
  // The guarded low branch uses the 1/Z statistic; the clipped link follows cfg.inv_stat.
  const bool inv = clip ? cfg.inv_stat != 0 : true;
  int s;
#define ALGX_BWD(NN, CC, II) \
  launch_bwd<NN, CC, II>(maps[0], maps[1], maps[2], maps[3], cfg, stat, di, guard, acc, dk, dv, B, H, T, st)
  if (cfg.n == 16)
    s = clip ? (inv ? ALGX_BWD(16, true, true) : ALGX_BWD(16, true, false)) : ALGX_BWD(16, false, true);
  else if (cfg.n == 8)
    s = clip ? (inv ? ALGX_BWD(8, true, true) : ALGX_BWD(8, true, false)) : ALGX_BWD(8, false, true);
  else
    s = clip ? (inv ? ALGX_BWD(32, true, true) : ALGX_BWD(32, true, false)) : ALGX_BWD(32, false, true);
#undef ALGX_BWD
  if (s) return s;
  const int64_t n4 = (int64_t)(nacc / 4);
  const int grid = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 16);
  dq_finish_kernel<<<grid, 256, 0, st>>>(cfg, guard, reinterpret_cast<const float4*>(acc),
                                          static_cast<__nv_bfloat16*>(dq), n4);
  ALGX_LAUNCHED("dq_finish launch");
  *launched = true;
  return ALGX_OK;
}

}  // namespace algx
