// Fused LM head + likelihood (kernels/fused_head.py:72-216): logits
// z = h E^T never reach HBM.
//
// Forward (fused_head.py:72-117): CTA = (128-token block, vocabulary split).
// A TMA warp streams 64-wide K chunks of h and of 256-row E tiles through a
// 4-stage ring; one thread issues tcgen05 MMAs into two TMEM accumulators
// (128 x 256 fp32 each, double-buffered); 4 epilogue warps (thread = token)
// fold each tile into running statistics: online max / sum-exp for "ce",
// the additive sum of rho(min(z/c, X))^n for "alg_ce", and the target logit
// by column compare. Per-split partials are combined by algx_head_reduce and
// finished by algx_head_finalize (stat, telemetry, objective).
//
// Backward (fused_head.py:120-156, 194-216): two launches of one kernel.
// Mode 0 (dh): rows = tokens, columns = vocabulary; mode 1 (dE): rows =
// vocabulary, columns = tokens. A CTA owns 128 rows and one d-chunk (<= 256
// columns) of the output. Per 128-column tile it recomputes the logit tile
// (K loop over d), turns it into dz (softmax - y, or (p - y) r) scaled and
// rounded to bf16, stores dz into TMEM, and accumulates out += dz . Y[:, chunk]
// with dz as the TMEM A operand. dz is never written to HBM.
#include <algorithm>

#include "algx_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace algx {
namespace {

using namespace sm100;

constexpr int kRowsT = 128;
constexpr int kChunkBytes = 128 * 64 * 2;  // 128 rows x 64 bf16, one SW128 box

// ------------------------------------------------------------------ forward
constexpr int kFwdNT = 256;     // vocabulary columns per tile
constexpr int kFwdStages = 4;
constexpr int kFwdStageBytes = kChunkBytes + kFwdNT * 64 * 2;  // h chunk + E chunk
constexpr int kFwdSmem = kFwdStages * kFwdStageBytes + 1024;
constexpr int kHeadThreads = 192;

__device__ __forceinline__ uint8_t* align1k(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

struct HeadArgs {
  algx_head_config cfg;
  const int32_t* targets;
  int N;         // tokens
  int d;         // model width
  int V;         // local vocabulary rows
  int voff;      // global index of local row 0
  int splits;    // forward vocabulary splits
};

template <int KIND, int NPOW>
__global__ void __launch_bounds__(kHeadThreads, 1)
    head_fwd_tc_kernel(const __grid_constant__ CUtensorMap th, const __grid_constant__ CUtensorMap te, HeadArgs a,
                       float* __restrict__ part_m, float* __restrict__ part_l, float* __restrict__ part_zt,
                       int* dev_err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  __shared__ uint64_t full[kFwdStages], empty[kFwdStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tb = blockIdx.x, split = blockIdx.y;
  const int ntiles = (a.V + kFwdNT - 1) / kFwdNT;
  const int per = (ntiles + a.splits - 1) / a.splits;
  const int t0 = split * per, t1 = min(ntiles, t0 + per);
  const int nk = a.d / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 4) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp == 4) {
    if (lane == 0 && t0 < t1) {
      prefetch_tmap(&th);
      prefetch_tmap(&te);
      int it = 0;
      int last_stage_it[kFwdStages] = {-1, -1, -1, -1};
      for (int t = t0; t < t1 && !*abort_v; ++t)
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kFwdStages;
          if (it >= kFwdStages && !mbar_wait(&empty[s], ((it / kFwdStages) - 1) & 1, abort_v, dev_err)) break;
          uint8_t* st = smem + s * kFwdStageBytes;
          mbar_expect_tx(&full[s], kFwdStageBytes);
          tma_load_2d(st, &th, &full[s], kc * 64, tb * kRowsT);
          tma_load_2d(st + kChunkBytes, &te, &full[s], kc * 64, t * kFwdNT);
          last_stage_it[s] = it;
        }
      if (*abort_v)
        for (int s = 0; s < kFwdStages; ++s)
          if (last_stage_it[s] >= 0) {
            volatile int quiet = 0;
            mbar_wait(&full[s], (last_stage_it[s] / kFwdStages) & 1, &quiet, nullptr);
          }
    }
  } else if (warp == 5) {
    if (lane == 0 && t0 < t1) {
      const uint32_t id = idesc_bf16_f32(128, kFwdNT, 0, 0);
      const uint32_t s0 = smem_u32(smem);
      int it = 0;
      bool ok = true;
      for (int t = t0; ok && t < t1; ++t) {
        const int buf = (t - t0) & 1, use = (t - t0) >> 1;
        if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * kFwdNT;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kFwdStages;
          if (!mbar_wait(&full[s], (it / kFwdStages) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t hb = s0 + s * kFwdStageBytes, eb = hb + kChunkBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ss(acc, desc_sw128(hb + k * 32, 16, 1024), desc_sw128(eb + k * 32, 16, 1024), id, (kc > 0 || k > 0));
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // epilogue: thread r owns token tb*128 + r
    const int r = threadIdx.x;
    const int tok = tb * kRowsT + r;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const int tgt = tok < a.N ? a.targets[tok] : -2147483647 - 1;
    const int tloc = tgt - a.voff;  // local column of the target, may be out of range
    float m = -1e30f, l = 0.f, zt = 0.f;
    const float log2e = 1.4426950408889634f;
    for (int t = t0; t < t1; ++t) {
      const int buf = (t - t0) & 1, use = (t - t0) >> 1;
      if (!mbar_wait_warp(&acc_full[buf], use & 1, abort_v, dev_err)) break;
      tc_fence_after();
      const uint32_t acc = tmem_base + buf * kFwdNT + lane_off;
      const int cbase = t * kFwdNT;
#pragma unroll 1
      for (int c = 0; c < kFwdNT / 32; ++c) {
        uint32_t zr[32];
        tmem_ld32(acc + c * 32, zr);
        const int col0 = cbase + c * 32;
        const int nvalid = min(32, a.V - col0);
        if (tloc >= col0 && tloc < col0 + 32 && tloc < a.V) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col0 + i == tloc) zt += __uint_as_float(zr[i]);
        }
        if constexpr (KIND == ALGX_HEAD_CE) {
          float cm = -1e30f;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nvalid) cm = fmaxf(cm, __uint_as_float(zr[i]));
          if (cm > m) {
            l *= exp2f((m - cm) * log2e);
            m = cm;
          }
          const float mb = m * log2e;
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < nvalid) s += exp2f(fmaf(__uint_as_float(zr[i]), log2e, -mb));
          l += s;
        } else {
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i < nvalid) {
              const float x = fminf(__uint_as_float(zr[i]) * a.cfg.inv_c, a.cfg.clamp);
              const float rad = fmaf(x, x, 1.f);
              s += ipow_t<NPOW>(fmaf(rad, rsqrt_fast(rad), x));
            }
          }
          l += s;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (tok < a.N) {
      const size_t o = (size_t)split * a.N + tok;
      part_m[o] = m;
      part_l[o] = l;
      part_zt[o] = zt;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ backward
constexpr int kGradStages = 3;
constexpr int kGradStageBytes = 2 * kChunkBytes;  // X chunk + Y chunk (128 rows each)
constexpr int kGradThreads = 192;

struct GradArgs {
  algx_head_config cfg;
  const int32_t* targets;
  const float* stat;    // per token
  const float* scale;   // device scalar: g * slope / count
  int N, d, V, voff;
  int rows, cols;       // rows / columns of this launch (tokens or vocabulary)
  int dc;               // output d-chunk width (64..256, divides d)
  int out_bf16;         // output dtype
};

template <int MODE, int KIND, int NPOW>
__global__ void __launch_bounds__(kGradThreads, 1)
    head_grad_tc_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap ty, GradArgs a,
                        void* __restrict__ out, int* dev_err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  uint8_t* yout = smem + kGradStages * kGradStageBytes;         // [dc/64 boxes][128 rows][64]
  __shared__ uint64_t full[kGradStages], empty[kGradStages];
  __shared__ uint64_t z_full, dz_full, dz_free, yo_full, yo_empty, acc_done;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x, chunk = blockIdx.y;
  const int nk = a.d / 64;
  const int nct = (a.cols + 127) / 128;
  const int nbox = a.dc / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGradStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&z_full, 1);
    mbar_init(&dz_full, 4);
    mbar_init(&dz_free, 1);
    mbar_init(&yo_full, 1);
    mbar_init(&yo_empty, 1);
    mbar_init(&acc_done, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 4) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tZ = tmem_base, tDZ = tmem_base + 128, tACC = tmem_base + 256;

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tmap(&tx);
      prefetch_tmap(&ty);
      int it = 0;
      bool ok = true;
      for (int ct = 0; ok && ct < nct; ++ct) {
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kGradStages;
          if (it >= kGradStages && !mbar_wait(&empty[s], ((it / kGradStages) - 1) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kGradStageBytes;
          mbar_expect_tx(&full[s], kGradStageBytes);
          tma_load_2d(st, &tx, &full[s], kc * 64, rb * kRowsT);
          tma_load_2d(st + kChunkBytes, &ty, &full[s], kc * 64, ct * 128);
        }
        if (!ok) break;
        if (ct > 0 && !mbar_wait(&yo_empty, (ct - 1) & 1, abort_v, dev_err)) break;
        mbar_expect_tx(&yo_full, nbox * kChunkBytes);
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(yout + bx * kChunkBytes, &ty, &yo_full, chunk * a.dc + bx * 64, ct * 128);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t idz = idesc_bf16_f32(128, 128, 0, 0);
      const uint32_t ido = idesc_bf16_f32(128, a.dc, 0, 1);
      const uint32_t s0 = smem_u32(smem), y0 = smem_u32(yout);
      int it = 0;
      bool ok = true;
      auto out_mma = [&](int ct) -> bool {
        if (!mbar_wait(&dz_full, ct & 1, abort_v, dev_err)) return false;
        if (!mbar_wait(&yo_full, ct & 1, abort_v, dev_err)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_ts(tACC, tDZ + k * 8, desc_sw128(y0 + k * 2048, kChunkBytes, 1024), ido, (ct > 0 || k > 0));
        mma_commit(&dz_free);
        mma_commit(&yo_empty);
        return true;
      };
      for (int ct = 0; ok && ct < nct; ++ct) {
        // the z buffer is free once the epilogue has turned z_{ct-1} into dz
        if (ct > 0 && !out_mma(ct - 1)) break;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kGradStages;
          if (!mbar_wait(&full[s], (it / kGradStages) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xb = s0 + s * kGradStageBytes, yb = xb + kChunkBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ss(tZ, desc_sw128(xb + k * 32, 16, 1024), desc_sw128(yb + k * 32, 16, 1024), idz, (kc > 0 || k > 0));
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&z_full);
      }
      if (ok && !*abort_v && out_mma(nct - 1)) mma_commit(&acc_done);
    }
  } else {
    const int r = threadIdx.x;
    const int row = rb * kRowsT + r;  // token (mode 0) or local vocabulary row (mode 1)
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const algx_head_config& c = a.cfg;
    const float scale = *a.scale;
    // mode 0: per-row token statistics
    float rstat = 0.f;
    int rtgt = 0;
    bool rvalid = row < a.rows;
    if (MODE == 0 && rvalid) {
      rstat = a.stat[row];
      rtgt = a.targets[row];
      if (c.has_ignore && rtgt == c.ignore_index) rvalid = false;
    }
    const int vrow = row + a.voff;  // mode 1: global vocabulary index of this row
    bool ok = true;
    for (int ct = 0; ct < nct; ++ct) {
      if (!mbar_wait_warp(&z_full, ct & 1, abort_v, dev_err)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t zr[32];
        tmem_ld32(tZ + lane_off + cc * 32, zr);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float dzv[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int jj = cc * 32 + 2 * i + h;      // column within the tile
            const int col = ct * 128 + jj;          // token (mode 1) or local vocab (mode 0)
            const float z = __uint_as_float(zr[2 * i + h]);
            float st, y;
            bool valid;
            if (MODE == 0) {
              valid = rvalid && col < a.cols;
              st = rstat;
              y = (col + a.voff == rtgt) ? 1.f : 0.f;
            } else {
              // token statistics of column col (the same address in every
              // lane: one broadcast load)
              const bool in = col < a.N;
              const int tg = in ? __ldg(a.targets + col) : 0;
              valid = row < a.rows && in && !(c.has_ignore && tg == c.ignore_index);
              st = in ? __ldg(a.stat + col) : 0.f;
              y = (vrow == tg) ? 1.f : 0.f;
            }
            float g;
            if constexpr (KIND == ALGX_HEAD_CE) {
              g = __expf(z - st) - y;
            } else {
              const float x = fminf(z * c.inv_c, c.clamp);
              const float rad = fmaf(x, x, 1.f);
              const float rr = rsqrt_fast(rad);
              g = (ipow_t<NPOW>(fmaf(rad, rr, x) * st) - y) * rr;
            }
            dzv[h] = valid ? g * scale : 0.f;
          }
          pk[i] = pack_bf16x2(dzv[0], dzv[1]);
        }
        if (cc == 0 && ct > 0 && !mbar_wait_warp(&dz_free, (ct - 1) & 1, abort_v, dev_err)) {
          ok = false;
          break;
        }
        tmem_st16(tDZ + lane_off + cc * 16, pk);
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dz_full);
    }
    // The TMEM loads are warp-collective: every lane reads, only rows in
    // range store.
    if (ok && mbar_wait_warp(&acc_done, 0, abort_v, dev_err)) {
      tc_fence_after();
      const bool store = row < a.rows;
      for (int c0 = 0; c0 < a.dc; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tACC + lane_off + c0, v);
        if (!store) continue;
        const size_t o = (size_t)row * a.d + (size_t)chunk * a.dc + c0;
        if (a.out_bf16) {
          uint4* d4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + o);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            d4[u] = make_uint4(pack_bf16x2(__uint_as_float(v[8 * u]), __uint_as_float(v[8 * u + 1])),
                               pack_bf16x2(__uint_as_float(v[8 * u + 2]), __uint_as_float(v[8 * u + 3])),
                               pack_bf16x2(__uint_as_float(v[8 * u + 4]), __uint_as_float(v[8 * u + 5])),
                               pack_bf16x2(__uint_as_float(v[8 * u + 6]), __uint_as_float(v[8 * u + 7])));
        } else {
          float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
#pragma unroll
          for (int u = 0; u < 8; ++u)
            d4[u] = make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                                __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) tmem_dealloc(tmem_base, 512);
}

// ------------------------------------------------------------------ statistics
// Combine `splits` forward partials per token: max/rescaled sum (ce) or sum (alg_ce).
__global__ void head_reduce_kernel(algx_head_config cfg, const float* __restrict__ pm, const float* __restrict__ pl,
                                   const float* __restrict__ pz, int splits, int N, float* __restrict__ m,
                                   float* __restrict__ l, float* __restrict__ zt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  float mm = -1e30f, ll = 0.f, zz = 0.f;
  if (cfg.kind == ALGX_HEAD_CE) {
    for (int s = 0; s < splits; ++s) mm = fmaxf(mm, pm[(size_t)s * N + i]);
    for (int s = 0; s < splits; ++s) ll += pl[(size_t)s * N + i] * __expf(pm[(size_t)s * N + i] - mm);
  } else {
    for (int s = 0; s < splits; ++s) ll += pl[(size_t)s * N + i];
  }
  for (int s = 0; s < splits; ++s) zz += pz[(size_t)s * N + i];
  m[i] = mm;
  l[i] = ll;
  zt[i] = zz;
}

// stat, telemetry and objective (fused_head.py:219-229), with the optional
// ignore_index: ignored rows get telemetry 0 and leave the mean. One CTA,
// fixed-order reduction; writes obj[0] and count[0].
__global__ void __launch_bounds__(1024) head_finalize_kernel(algx_head_config cfg, const int32_t* __restrict__ targets,
                                                             const float* __restrict__ m, const float* __restrict__ l,
                                                             const float* __restrict__ zt, int N, int V_total,
                                                             float* __restrict__ stat, float* __restrict__ tel,
                                                             float* __restrict__ obj, float* __restrict__ count,
                                                             int* dev_err) {
  __shared__ float red_s[1024];
  __shared__ float red_c[1024];
  float s = 0.f, cnt = 0.f;
  int bad = 0;
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    const int t = targets[i];
    const bool ignored = cfg.has_ignore && t == cfg.ignore_index;
    if (cfg.has_ignore && !ignored && (t < 0 || t >= V_total)) bad = 1;
    float st, te;
    if (cfg.kind == ALGX_HEAD_CE) {
      st = m[i] + logf(l[i]);
      te = st - zt[i];
    } else {
      st = inv_root(l[i], cfg.n);
      const float x = fminf(zt[i] * cfg.inv_c, cfg.clamp);
      float r;
      te = ipow(rho_exact(x, r) * st, cfg.n);
    }
    stat[i] = st;
    if (ignored) {
      tel[i] = 0.f;
    } else {
      tel[i] = te;
      s += cfg.kind == ALGX_HEAD_CE ? te : 1.f - te;
      cnt += 1.f;
    }
  }
  if (bad && dev_err) atomicOr(dev_err, DEV_ERR_BAD_LABEL);
  red_s[threadIdx.x] = s;
  red_c[threadIdx.x] = cnt;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      red_s[threadIdx.x] += red_s[threadIdx.x + w];
      red_c[threadIdx.x] += red_c[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float n = cfg.has_ignore ? fmaxf(red_c[0], 1.f) : (float)N;
    obj[0] = red_s[0] / n;
    count[0] = n;
  }
}

int check_head(const algx_head_config* cfg, int64_t N, int64_t d, int64_t V, int32_t dtype) {
  ALGX_REQUIRE(cfg, "head: NULL config");
  ALGX_REQUIRE(cfg->kind == ALGX_HEAD_CE || cfg->kind == ALGX_HEAD_ALG_CE, "head: kind must be ce or alg_ce");
  if (cfg->kind == ALGX_HEAD_ALG_CE)
    ALGX_REQUIRE(cfg->n == 2 || cfg->n == 4 || cfg->n == 8 || cfg->n == 16 || cfg->n == 32,
                 "head: alg_ce power must be 2, 4, 8, 16 or 32");
  ALGX_REQUIRE(dtype == ALGX_BF16, "head: the tensor-core path takes bfloat16 h and embedding");
  ALGX_REQUIRE(N >= 1 && N <= (1ll << 30), "head: token count out of range");
  ALGX_REQUIRE(d >= 64 && d % 64 == 0 && d <= 16384, "head: d must be a positive multiple of 64");
  ALGX_REQUIRE(V >= 1 && V <= (1ll << 30), "head: vocabulary out of range");
  return ALGX_OK;
}

template <int KIND>
int launch_fwd_k(const CUtensorMap& th, const CUtensorMap& te, const HeadArgs& a, int tb, float* pm, float* pl,
                 float* pz, cudaStream_t st) {
  auto run = [&](auto kern) -> int {
    ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
    kern<<<dim3(tb, a.splits), kHeadThreads, kFwdSmem, st>>>(th, te, a, pm, pl, pz, device_error_word());
    ALGX_LAUNCHED("head_fwd_tc launch");
    return ALGX_OK;
  };
  if (KIND == ALGX_HEAD_CE) return run(head_fwd_tc_kernel<ALGX_HEAD_CE, 1>);
  switch (a.cfg.n) {
    case 2: return run(head_fwd_tc_kernel<ALGX_HEAD_ALG_CE, 2>);
    case 4: return run(head_fwd_tc_kernel<ALGX_HEAD_ALG_CE, 4>);
    case 8: return run(head_fwd_tc_kernel<ALGX_HEAD_ALG_CE, 8>);
    case 16: return run(head_fwd_tc_kernel<ALGX_HEAD_ALG_CE, 16>);
    default: return run(head_fwd_tc_kernel<ALGX_HEAD_ALG_CE, 32>);
  }
}

template <int MODE, int KIND>
int launch_grad_k(const CUtensorMap& tx, const CUtensorMap& ty, const GradArgs& a, void* out, cudaStream_t st) {
  const int smem = kGradStages * kGradStageBytes + 4 * kChunkBytes + 1024;
  const dim3 grid((unsigned)((a.rows + 127) / 128), (unsigned)(a.d / a.dc));
  auto run = [&](auto kern) -> int {
    ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kern<<<grid, kGradThreads, smem, st>>>(tx, ty, a, out, device_error_word());
    ALGX_LAUNCHED("head_grad_tc launch");
    return ALGX_OK;
  };
  if (KIND == ALGX_HEAD_CE) return run(head_grad_tc_kernel<MODE, ALGX_HEAD_CE, 1>);
  switch (a.cfg.n) {
    case 2: return run(head_grad_tc_kernel<MODE, ALGX_HEAD_ALG_CE, 2>);
    case 4: return run(head_grad_tc_kernel<MODE, ALGX_HEAD_ALG_CE, 4>);
    case 8: return run(head_grad_tc_kernel<MODE, ALGX_HEAD_ALG_CE, 8>);
    case 16: return run(head_grad_tc_kernel<MODE, ALGX_HEAD_ALG_CE, 16>);
    default: return run(head_grad_tc_kernel<MODE, ALGX_HEAD_ALG_CE, 32>);
  }
}

int pick_chunk(int64_t d) {
  for (int c : {256, 192, 128, 64})
    if (d % c == 0) return c;
  return 64;
}

}  // namespace
}  // namespace algx

using namespace algx;

extern "C" {

int algx_head_fwd_splits(int64_t N, int64_t V) {
  const int64_t tb = (N + 127) / 128, nt = (V + kFwdNT - 1) / kFwdNT;
  int64_t s = (2 * 148 + tb - 1) / tb;
  if (s < 1) s = 1;
  if (s > nt) s = nt;
  if (s > 64) s = 64;
  return (int)s;
}

int algx_head_fwd(const algx_head_config* cfg, const void* h, const void* embed, const int32_t* targets,
                  float* part_m, float* part_l, float* part_zt, int64_t N, int64_t d, int64_t V, int64_t vocab_offset,
                  int32_t splits, int32_t dtype, void* stream) {
  if (int s = check_head(cfg, N, d, V, dtype)) return s;
  ALGX_REQUIRE(h && embed && targets && part_m && part_l && part_zt, "head_fwd: NULL pointer");
  ALGX_REQUIRE(splits >= 1 && splits <= 64, "head_fwd: splits must be in [1, 64]");
  CUtensorMap th, te;
  if (int s = make_tmap_2d(&th, h, ALGX_BF16, (uint64_t)d, (uint64_t)N, (uint64_t)d * 2, 64, 128, true)) return s;
  if (int s = make_tmap_2d(&te, embed, ALGX_BF16, (uint64_t)d, (uint64_t)V, (uint64_t)d * 2, 64, kFwdNT, true))
    return s;
  HeadArgs a{*cfg, targets, (int)N, (int)d, (int)V, (int)vocab_offset, splits};
  const int tb = (int)((N + 127) / 128);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return cfg->kind == ALGX_HEAD_CE ? launch_fwd_k<ALGX_HEAD_CE>(th, te, a, tb, part_m, part_l, part_zt, st)
                                   : launch_fwd_k<ALGX_HEAD_ALG_CE>(th, te, a, tb, part_m, part_l, part_zt, st);
}

int algx_head_reduce(const algx_head_config* cfg, const float* part_m, const float* part_l, const float* part_zt,
                     int32_t splits, int64_t N, float* m, float* l, float* zt, void* stream) {
  ALGX_REQUIRE(cfg && part_m && part_l && part_zt && m && l && zt, "head_reduce: NULL pointer");
  ALGX_REQUIRE(N >= 1 && splits >= 1, "head_reduce: empty input");
  head_reduce_kernel<<<(unsigned)((N + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      *cfg, part_m, part_l, part_zt, splits, (int)N, m, l, zt);
  ALGX_LAUNCHED("head_reduce launch");
  return ALGX_OK;
}

int algx_head_finalize(const algx_head_config* cfg, const int32_t* targets, const float* m, const float* l,
                       const float* zt, int64_t N, int64_t V_total, float* stat, float* telemetry, float* objective,
                       float* count, void* stream) {
  ALGX_REQUIRE(cfg && targets && m && l && zt && stat && telemetry && objective && count,
               "head_finalize: NULL pointer");
  ALGX_REQUIRE(N >= 1, "head_finalize: empty input");
  head_finalize_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      *cfg, targets, m, l, zt, (int)N, (int)V_total, stat, telemetry, objective, count, device_error_word());
  ALGX_LAUNCHED("head_finalize launch");
  return ALGX_OK;
}

int algx_head_bwd(const algx_head_config* cfg, const void* h, const void* embed, const int32_t* targets,
                  const float* stat, const float* scale, void* dh, int32_t dh_dtype, float* dembed, int64_t N,
                  int64_t d, int64_t V, int64_t vocab_offset, int32_t dtype, void* stream) {
  if (int s = check_head(cfg, N, d, V, dtype)) return s;
  ALGX_REQUIRE(h && embed && targets && stat && scale && dh && dembed, "head_bwd: NULL pointer");
  ALGX_REQUIRE(dh_dtype == ALGX_F32 || dh_dtype == ALGX_BF16, "head_bwd: dh dtype must be float32 or bfloat16");
  CUtensorMap th, te;
  if (int s = make_tmap_2d(&th, h, ALGX_BF16, (uint64_t)d, (uint64_t)N, (uint64_t)d * 2, 64, 128, true)) return s;
  if (int s = make_tmap_2d(&te, embed, ALGX_BF16, (uint64_t)d, (uint64_t)V, (uint64_t)d * 2, 64, 128, true))
    return s;
  GradArgs a{*cfg, targets, stat, scale, (int)N, (int)d, (int)V, (int)vocab_offset, 0, 0, pick_chunk(d), 0};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // dh: rows = tokens, columns = vocabulary
  GradArgs ah = a;
  ah.rows = (int)N;
  ah.cols = (int)V;
  ah.out_bf16 = dh_dtype == ALGX_BF16;
  int s = cfg->kind == ALGX_HEAD_CE ? launch_grad_k<0, ALGX_HEAD_CE>(th, te, ah, dh, st)
                                    : launch_grad_k<0, ALGX_HEAD_ALG_CE>(th, te, ah, dh, st);
  if (s) return s;
  // dE: rows = vocabulary, columns = tokens
  GradArgs ae = a;
  ae.rows = (int)V;
  ae.cols = (int)N;
  ae.out_bf16 = 0;
  return cfg->kind == ALGX_HEAD_CE ? launch_grad_k<1, ALGX_HEAD_CE>(te, th, ae, dembed, st)
                                   : launch_grad_k<1, ALGX_HEAD_ALG_CE>(te, th, ae, dembed, st);
}

}  // extern "C"
