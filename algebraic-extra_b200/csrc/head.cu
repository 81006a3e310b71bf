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
// Backward (fused_head.py:120-156, 194-216), one vocabulary slab of
// kSlabCols columns at a time, so the logits are never materialised in full:
// head_dz_tc_kernel recomputes the slab's logits with the forward's pipeline
// and its epilogue writes dz = (softmax - y) or (p - y) r, scaled and rounded
// to bf16 (the reference's dzb), into a slab-sized workspace; head_gemm_pair_kernel
// then consumes the slab with both products on tcgen05 tensor cores in one
// persistent launch: dE_slab = dz^T . h and dh += dz . E_slab (fp32
// accumulation across slabs by TMA reduce-adds). The slab width sets how
// evenly the GEMM's tiles (dE tiles with the whole token reduction, four to
// six times the work of a dh tile) fill 148 SMs: at config 3, 6656 columns
// (8 slabs of 16384 x 6656 bf16, 218 MB) leave the last wave of each launch
// ~95% full where 4096 columns (13 slabs) left ~84%; the dz slab then exceeds
// L2, and the GEMM's second read of it comes partly from HBM, well within
// the tensor-bound launch's bandwidth.
#include <algorithm>
#include <string>

#include "algx_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace algx {
namespace {

using namespace sm100;

constexpr int kRowsT = 128;
constexpr int kChunkBytes = 128 * 64 * 2;  // 128 rows x 64 bf16, one SW128 box

// ------------------------------------------------------------------ forward
// The forward and the dz recompute run on CTA pairs (clusters of two,
// cta_group::2), like the slab GEMM: a pair computes 256 tokens x 256
// vocabulary columns per tile with M = 256 products issued by the leader
// (cluster rank 0); CTA r holds token rows 128 r.. (its own TMEM lanes) and
// loads its 128 tokens of h and 128 of the tile's 256 E rows per 64-wide K
// chunk, both CTAs' loads completing on the leader's stage barrier. Each
// CTA's epilogue reads its 128 rows x 256 columns of the accumulator.
constexpr int kFwdNT = 256;     // vocabulary columns per tile
constexpr int kFwdStages = 6;
constexpr int kFwdStageBytes = kChunkBytes + 128 * 64 * 2;  // this CTA's h chunk + half of the E chunk
constexpr int kFwdSmem = kFwdStages * kFwdStageBytes + 1024;
// dz kernel: the load ring plus one 16 KB staging box per epilogue group
// (128 token rows x 64 bf16 columns, 128-byte swizzle) for its TMA stores
constexpr int kDzBoxBytes = 128 * 64 * 2;
constexpr int kDzSmem = kFwdSmem + 2 * kDzBoxBytes;
static_assert(kDzSmem <= 227 * 1024, "dz kernel shared memory");
constexpr int kHeadThreads = 320;  // 2 x 4 epilogue warps, TMA warp, MMA warp
constexpr int kHeadTma = 8;

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

// Maximum of 32 fp32 values (raw bits) by a tree of depth 5.
__device__ __forceinline__ float chunk_max32(const uint32_t (&zr)[32]) {
  float mx[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) mx[i] = fmaxf(__uint_as_float(zr[2 * i]), __uint_as_float(zr[2 * i + 1]));
#pragma unroll
  for (int w = 8; w > 0; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
  return mx[0];
}

template <int KIND, int NPOW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kHeadThreads, 1)
    head_fwd_tc_kernel(const __grid_constant__ CUtensorMap th, const __grid_constant__ CUtensorMap te, HeadArgs a,
                       float* __restrict__ part_m, float* __restrict__ part_l, float* __restrict__ part_zt,
                       int* dev_err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  __shared__ uint64_t full[kFwdStages], empty[kFwdStages], acc_full[2], acc_empty[2], x_ready, issued;
  __shared__ float xm[kRowsT], xl[kRowsT], xz[kRowsT];  // statistics of epilogue group 1
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tb = blockIdx.x, split = blockIdx.y;  // pairs are consecutive token blocks
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
      mbar_init(&acc_empty[b], 8);  // four epilogue warps of each CTA of the pair
    }
    mbar_init(&x_ready, 4);
    mbar_init(&issued, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == kHeadTma) {  // the same warp of both CTAs allocates the pair's TMEM
    tmem_alloc_pair(&tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t full0 = cluster_addr(&full[0], 0);

  if (warp == kHeadTma) {
    if (lane == 0 && t0 < t1) {
      prefetch_tmap(&th);
      prefetch_tmap(&te);
      int it = 0;
      int last_stage_it[kFwdStages] = {-1, -1, -1, -1};
      for (int t = t0; t < t1 && !*abort_v; ++t)
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kFwdStages;
          if (it >= kFwdStages && !mbar_wait_cluster(&empty[s], ((it / kFwdStages) - 1) & 1, abort_v, dev_err))
            break;
          uint8_t* st = smem + s * kFwdStageBytes;
          if (leader) mbar_expect_tx(&full[s], 2 * kFwdStageBytes);  // both CTAs' halves
          tma_load_2d_pair(st, &th, full0 + s * 8, kc * 64, tb * kRowsT);
          tma_load_2d_pair(st + kChunkBytes, &te, full0 + s * 8, kc * 64, t * kFwdNT + 128 * (int)rank);
          last_stage_it[s] = it;
        }
      if (*abort_v && leader)
        for (int s = 0; s < kFwdStages; ++s)
          if (last_stage_it[s] >= 0) {
            volatile int quiet = 0;
            mbar_wait_cluster(&full[s], (last_stage_it[s] / kFwdStages) & 1, &quiet, nullptr);
          }
    }
  } else if (warp == kHeadTma + 1) {
    if (lane == 0 && t0 < t1 && leader) {
      const uint32_t id = idesc_bf16_f32(256, kFwdNT, 0, 0);
      const uint32_t empty0 = cluster_addr(&empty[0], 0), empty1 = cluster_addr(&empty[0], 1);
      const uint32_t accf0 = cluster_addr(&acc_full[0], 0), accf1 = cluster_addr(&acc_full[0], 1);
      const uint32_t s0 = smem_u32(smem);
      int it = 0;
      bool ok = true;
      for (int t = t0; ok && t < t1; ++t) {
        const int buf = (t - t0) & 1, use = (t - t0) >> 1;
        if (use > 0 && !mbar_wait_cluster(&acc_empty[buf], (use - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * kFwdNT;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kFwdStages;
          if (!mbar_wait_cluster(&full[s], (it / kFwdStages) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t hb = s0 + s * kFwdStageBytes, eb = hb + kChunkBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ss_pair(acc, desc_sw128(hb + k * 32, 16, 1024), desc_sw128(eb + k * 32, 16, 1024), id,
                        (kc > 0 || k > 0));
          mma_commit_pair(empty0 + s * 8);  // the stage is free again in both CTAs
          mma_commit_pair(empty1 + s * 8);
        }
        if (ok) {
          mma_commit_pair(accf0 + buf * 8);
          mma_commit_pair(accf1 + buf * 8);
        }
      }
      mma_commit_pair(cluster_addr(&issued, 0));  // settle before TMEM is freed
      volatile int quiet = 0;
      mbar_wait_cluster(&issued, 0, &quiet, dev_err);
    }
  } else {
    // epilogue: two groups of four warps take alternate tiles (group g owns
    // accumulator buffer g); thread r of a group owns token tb*128 + r
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int tok = tb * kRowsT + r;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int tgt = tok < a.N ? a.targets[tok] : -2147483647 - 1;
    const int tloc = tgt - a.voff;  // local column of the target, may be out of range
    float m = -1e30f, l = 0.f, zt = 0.f;
    const float log2e = 1.4426950408889634f;
    for (int t = t0 + g; t < t1; t += 2) {
      const int buf = g, use = (t - t0) >> 1;
      if (!mbar_wait_cluster_warp(&acc_full[buf], use & 1, abort_v, dev_err)) break;
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
        if (nvalid == 32) {
          // full chunk: the same per-element maths on packed f32x2 pairs with
          // two partial sums (and a max tree for ce), so a thread's 32
          // elements are not one serial dependency chain
          if constexpr (KIND == ALGX_HEAD_CE) {
            const float cm = chunk_max32(zr);
            if (cm > m) {
              l *= exp2f((m - cm) * log2e);
              m = cm;
            }
            const float2 lg = make_float2(log2e, log2e), nb = make_float2(-m * log2e, -m * log2e);
            float2 s0 = make_float2(0.f, 0.f), s1 = s0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 t = fma2(make_float2(__uint_as_float(zr[2 * i]), __uint_as_float(zr[2 * i + 1])), lg, nb);
              const float2 e = make_float2(exp2f(t.x), exp2f(t.y));
              if (i & 1) s1 = add2(s1, e);
              else s0 = add2(s0, e);
            }
            l += (s0.x + s0.y) + (s1.x + s1.y);
          } else {
            const float2 ic = make_float2(a.cfg.inv_c, a.cfg.inv_c), one = make_float2(1.f, 1.f);
            float2 s0 = make_float2(0.f, 0.f), s1 = s0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float2 x = mul2(make_float2(__uint_as_float(zr[2 * i]), __uint_as_float(zr[2 * i + 1])), ic);
              x.x = fminf(x.x, a.cfg.clamp);
              x.y = fminf(x.y, a.cfg.clamp);
              const float2 rad = fma2(x, x, one);
              const float2 rr = make_float2(rsqrt_fast(rad.x), rsqrt_fast(rad.y));
              const float2 p = ipow2_t<NPOW>(fma2(rad, rr, x));
              if (i & 1) s1 = add2(s1, p);
              else s0 = add2(s0, p);
            }
            l += (s0.x + s0.y) + (s1.x + s1.y);
          }
        } else if constexpr (KIND == ALGX_HEAD_CE) {
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
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&acc_empty[buf], 0));  // the leader's barrier
    }
    // group 1 hands its statistics to group 0, which merges and writes them
    if (g == 1) {
      xm[r] = m;
      xl[r] = l;
      xz[r] = zt;
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_ready);  // release: the row statistics are visible to group 0
    } else if (mbar_wait_warp(&x_ready, 0, abort_v, dev_err) && tok < a.N) {
      const float m1 = xm[r], l1 = xl[r];
      if constexpr (KIND == ALGX_HEAD_CE) {
        const float mm = fmaxf(m, m1);
        l = l * exp2f((m - mm) * log2e) + l1 * exp2f((m1 - mm) * log2e);
        m = mm;
      } else {
        l += l1;
      }
      zt += xz[r];
      const size_t o = (size_t)split * a.N + tok;
      part_m[o] = m;
      part_l[o] = l;
      part_zt[o] = zt;
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's last products (which read this CTA's shared memory) are done
  tc_fence_after();
  if (warp == kHeadTma) tmem_dealloc_pair(tmem_base, 512);
}

// ------------------------------------------------------------------ backward
constexpr int kSlabCols = 6656;  // vocabulary columns per backward slab (26 forward tiles)

struct DzArgs {
  algx_head_config cfg;
  const int32_t* targets;
  const float* stat;   // per token
  const float* scale;  // device scalar: g * slope / count
  int N, d, V, voff;
  int tile0;           // first (local) vocabulary tile of the slab
  int ntiles;          // tiles in the slab
  int items;           // (256-token block, tile) work items of the slab: blocks x ntiles
  int* gemm_counter;   // tile counter of this slab's GEMM, zeroed here
};

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Logits of one slab with the forward's load / MMA pipeline; the epilogue
// (thread = token) turns each fp32 logit into bf16 dz and stores its row
// segment of the slab. Columns past the vocabulary and ignored rows give 0.
// Persistent: CTA pair p takes the work items p, p + pairs, ... (item i =
// 256-token block i / ntiles, tile i % ntiles; CTA r of the pair holds token
// block 2 (i / ntiles) + r), so the load ring and the two TMEM accumulators
// run on across items and every pair gets an equal share of the slab's items.
template <int KIND, int NPOW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kHeadThreads, 1)
    head_dz_tc_kernel(const __grid_constant__ CUtensorMap th, const __grid_constant__ CUtensorMap te,
                      const __grid_constant__ CUtensorMap tdz, DzArgs a, int* dev_err) {
  pdl_trigger();  // the slab's GEMM may be scheduled as this grid's CTAs finish
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  __shared__ uint64_t full[kFwdStages], empty[kFwdStages], acc_full[2], acc_empty[2], issued;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = a.d / 64;
  const int first = blockIdx.x >> 1, stride = gridDim.x >> 1;  // pair items

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // four epilogue warps of each CTA of the pair
    }
    mbar_init(&issued, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == kHeadTma) {  // the same warp of both CTAs allocates the pair's TMEM
    tmem_alloc_pair(&tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t full0 = cluster_addr(&full[0], 0);

  if (warp == kHeadTma) {
    if (lane == 0 && first < a.items) {
      prefetch_tmap(&th);
      prefetch_tmap(&te);
      int it = 0;
      int last_stage_it[kFwdStages] = {-1, -1, -1, -1};
      for (int i = first; i < a.items && !*abort_v; i += stride) {
        const int tb = 2 * (i / a.ntiles) + (int)rank, t = a.tile0 + i % a.ntiles;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kFwdStages;
          if (it >= kFwdStages && !mbar_wait_cluster(&empty[s], ((it / kFwdStages) - 1) & 1, abort_v, dev_err))
            break;
          uint8_t* st = smem + s * kFwdStageBytes;
          if (leader) mbar_expect_tx(&full[s], 2 * kFwdStageBytes);  // both CTAs' halves
          tma_load_2d_pair(st, &th, full0 + s * 8, kc * 64, tb * kRowsT);
          tma_load_2d_pair(st + kChunkBytes, &te, full0 + s * 8, kc * 64, t * kFwdNT + 128 * (int)rank);
          last_stage_it[s] = it;
        }
      }
      if (*abort_v && leader)
        for (int s = 0; s < kFwdStages; ++s)
          if (last_stage_it[s] >= 0) {
            volatile int quiet = 0;
            mbar_wait_cluster(&full[s], (last_stage_it[s] / kFwdStages) & 1, &quiet, nullptr);
          }
    }
  } else if (warp == kHeadTma + 1) {
    if (lane == 0 && first < a.items && leader) {
      const uint32_t id = idesc_bf16_f32(256, kFwdNT, 0, 0);
      const uint32_t empty0 = cluster_addr(&empty[0], 0), empty1 = cluster_addr(&empty[0], 1);
      const uint32_t accf0 = cluster_addr(&acc_full[0], 0), accf1 = cluster_addr(&acc_full[0], 1);
      const uint32_t s0 = smem_u32(smem);
      int it = 0;
      bool ok = true;
      for (int i = first, li = 0; ok && i < a.items; i += stride, ++li) {
        const int buf = li & 1, use = li >> 1;
        if (use > 0 && !mbar_wait_cluster(&acc_empty[buf], (use - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * kFwdNT;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % kFwdStages;
          if (!mbar_wait_cluster(&full[s], (it / kFwdStages) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t hb = s0 + s * kFwdStageBytes, eb = hb + kChunkBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_ss_pair(acc, desc_sw128(hb + k * 32, 16, 1024), desc_sw128(eb + k * 32, 16, 1024), id,
                        (kc > 0 || k > 0));
          mma_commit_pair(empty0 + s * 8);  // the stage is free again in both CTAs
          mma_commit_pair(empty1 + s * 8);
        }
        if (ok) {
          mma_commit_pair(accf0 + buf * 8);
          mma_commit_pair(accf1 + buf * 8);
        }
      }
      mma_commit_pair(cluster_addr(&issued, 0));  // settle before TMEM is freed
      volatile int quiet = 0;
      mbar_wait_cluster(&issued, 0, &quiet, dev_err);
    }
  } else {
    // epilogue: two groups of four warps take alternate items (group g owns
    // accumulator buffer g); thread r of a group owns row r of the item's
    // 128-token block
    // Launched as a programmatic dependent of the previous slab's GEMM, which
    // reads the dz buffer: the loads and products of the first items above
    // overlap its tail; the epilogue writes dz (and resets this slab's GEMM
    // counter, last used two slabs ago) only once it has finished. h, E and
    // the statistics were complete before the first slab's normal launch.
    pdl_wait();
    if (blockIdx.x == 0 && warp == 0 && lane == 0) *a.gemm_counter = 0;
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const algx_head_config& c = a.cfg;
    const float scale = *a.scale;
    const float log2e = 1.4426950408889634f;
    // dz leaves through the group's staging box: two 32-column chunks fill its
    // 128-byte rows (swizzled), then one thread stores the box with TMA
    // (whole 128-byte lines instead of 16-byte pieces of 32 different rows
    // per warp store; rows past N are clipped by the tensor map)
    uint8_t* box = smem + kFwdStages * kFwdStageBytes + g * kDzBoxBytes;
    const bool issuer = (warp & 3) == 0 && lane == 0;
    for (int i = first + g * stride, li = g; i < a.items; i += 2 * stride, li += 2) {
      const int tb = 2 * (i / a.ntiles) + (int)rank, t = a.tile0 + i % a.ntiles;
      const int tok = tb * kRowsT + r;
      const int tgt = tok < a.N ? a.targets[tok] : -2147483647 - 1;
      const bool row_ok = tok < a.N && !(c.has_ignore && tgt == c.ignore_index);
      const int tloc = tgt - a.voff;  // local column of the target, may be out of range
      const float st = tok < a.N ? a.stat[tok] : 0.f;
      const float stl = st * log2e;
      const int xcol = (t - a.tile0) * kFwdNT;  // the tile's first column in the slab buffer
      const int buf = g, use = li >> 1;
      if (!mbar_wait_cluster_warp(&acc_full[buf], use & 1, abort_v, dev_err)) break;
      tc_fence_after();
      const uint32_t acc = tmem_base + buf * kFwdNT + lane_off;
#pragma unroll 1
      for (int cc = 0; cc < kFwdNT / 32; ++cc) {
        uint32_t zr[32];
        tmem_ld32(acc + cc * 32, zr);
        const int col0 = t * kFwdNT + cc * 32;
        uint32_t pk[16];
        if (col0 + 32 <= a.V) {
          // whole chunk inside the vocabulary (the same for every thread of the
          // warp, so ignored rows do not split it between the two paths): the
          // same per-element maths on packed f32x2 pairs; rows that are ignored
          // or past the end select zero
          const float2 sc = make_float2(scale, scale);
#pragma unroll
          for (int i2 = 0; i2 < 16; ++i2) {
            const float2 z = make_float2(__uint_as_float(zr[2 * i2]), __uint_as_float(zr[2 * i2 + 1]));
            const float2 y = make_float2(col0 + 2 * i2 == tloc ? 1.f : 0.f, col0 + 2 * i2 + 1 == tloc ? 1.f : 0.f);
            float2 gr;
            if constexpr (KIND == ALGX_HEAD_CE) {
              const float2 u = fma2(z, make_float2(log2e, log2e), make_float2(-stl, -stl));
              gr = sub2(make_float2(exp2f(u.x), exp2f(u.y)), y);
            } else {
              float2 x = mul2(z, make_float2(c.inv_c, c.inv_c));
              x.x = fminf(x.x, c.clamp);
              x.y = fminf(x.y, c.clamp);
              const float2 rad = fma2(x, x, make_float2(1.f, 1.f));
              const float2 rr = make_float2(rsqrt_fast(rad.x), rsqrt_fast(rad.y));
              gr = mul2(sub2(ipow2_t<NPOW>(mul2(fma2(rad, rr, x), make_float2(st, st))), y), rr);
            }
            const float2 g2 = mul2(gr, sc);
            pk[i2] = row_ok ? pack_bf16x2(g2.x, g2.y) : 0u;
          }
        } else {
#pragma unroll
        for (int i2 = 0; i2 < 16; ++i2) {
          float g2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int col = col0 + 2 * i2 + h;
            const float z = __uint_as_float(zr[2 * i2 + h]);
            const float y = col == tloc ? 1.f : 0.f;
            float gr;
            if constexpr (KIND == ALGX_HEAD_CE) {
              gr = exp2f(fmaf(z, log2e, -stl)) - y;
            } else {
              const float x = fminf(z * c.inv_c, c.clamp);
              const float rad = fmaf(x, x, 1.f);
              const float rr = rsqrt_fast(rad);
              gr = (ipow_t<NPOW>(fmaf(rad, rr, x) * st) - y) * rr;
            }
            g2[h] = (row_ok && col < a.V) ? gr * scale : 0.f;
          }
          pk[i2] = pack_bf16x2(g2[0], g2[1]);
        }
        }
        const int half = cc & 1;
        if (!half) {  // the box's previous store has been read out of shared memory
          if (issuer) bulk_wait_group_read0();
          named_bar_sync(1 + g, 128);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(box + r * 128 + (((4 * half + u) ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        if (half) {
          fence_proxy_async_smem();
          named_bar_sync(1 + g, 128);
          if (issuer) {
            tma_store_2d(&tdz, box, xcol + (cc - 1) * 32, tb * kRowsT);
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&acc_empty[buf], 0));  // the leader's barrier
    }
    if (issuer) bulk_wait_group0();  // every store of this group has completed
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's last products (which read this CTA's shared memory) are done
  tc_fence_after();
  if (warp == kHeadTma) tmem_dealloc_pair(tmem_base, 512);
}

// ------------------------------------------------------------------ slab GEMM
// The two products of a backward slab on tcgen05 tensor cores, in one
// persistent launch:
//   problem 0: dE_slab (vc x d) = dz^T . h   (A = dz read MN-major, B = h MN-major, K = N tokens)
//   problem 1: dh (N x d) (+)= dz . E_slab  (A = dz K-major, B = E_slab MN-major, K = vc columns)
// Output tiles of 256 x 256 fp32 are handed out by a global counter, the large
// dE tiles (the whole token reduction) first and the dh tiles after them, so
// the CTA pairs that finish early take the remaining small tiles. A TMA warp
// streams 64-wide K chunks of A and B through a 6-stage ring; one thread
// issues the MMAs into two TMEM accumulators; two groups of four epilogue
// warps take alternate tiles and move each accumulator out in 32-column
// boxes (fp32, 128B-swizzled shared memory) with TMA stores, or TMA
// reduce-adds for dh after the first slab (the fp32 sum across slabs).
constexpr int kGemmBoxBytes = 128 * 32 * 4;  // epilogue staging box: 128 rows x 32 fp32
constexpr int kGemmThreads = 320;  // 2 x 4 epilogue warps, TMA warp, MMA warp

struct GemmProblem {
  int a_mn, b_mn;  // operand read MN-major (MN contiguous in memory) or K-major
  int add;         // epilogue: 0 = TMA store, 1 = TMA reduce-add
  int tiles_n;     // 256-column tiles of the output
  int tiles;       // output tiles
  int kchunks;     // 64-wide chunks of the reduction
};
struct GemmArgs {
  GemmProblem p[2];
  int* counter;  // zeroed by the slab's dz kernel
};

// The kernel runs on CTA pairs (cta_group::2): a cluster of two CTAs
// computes a 256 x 256 output tile with M = 256 products issued by the leader
// (cluster rank 0). CTA r loads A rows m0 + 128 r .. and B columns n0 + 128 r ..
// of each 64-wide K chunk into its own shared memory, so each SM reads and
// receives half of B per product instead of all of it: shared-memory traffic
// per product drops from ~192 to ~128 bytes per cycle, which is what bounds
// the one-CTA kernel near 0.65 of the tensor peak. Each CTA's TMEM holds its
// 128 rows of the two 256-column accumulators, and its epilogue writes them.
// Hand-offs between the CTAs: the leader's producer takes tiles from the
// global counter and publishes them in both CTAs' item queues; both CTAs'
// loads complete on the leader's stage barrier (the leader expects both
// halves' bytes); the leader's MMA thread frees each stage, and announces each
// accumulator, with one commit to each CTA's barrier; both epilogues release
// an accumulator by arriving on the leader's barrier.
constexpr int kPairBM = 256, kPairBN = 256, kPairStages = 6;
constexpr int kPairABytes = 128 * 64 * 2;  // this CTA's 128 rows of A x 64 K, 16 KB
constexpr int kPairBBytes = 128 * 64 * 2;  // this CTA's 128 columns of B x 64 K, 16 KB
constexpr int kPairStageBytes = kPairABytes + kPairBBytes;
constexpr int kPairSmem = kPairStages * kPairStageBytes + 2 * kGemmBoxBytes + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    head_gemm_pair_kernel(const __grid_constant__ CUtensorMap ta0, const __grid_constant__ CUtensorMap tb0,
                          const __grid_constant__ CUtensorMap tc0, const __grid_constant__ CUtensorMap ta1,
                          const __grid_constant__ CUtensorMap tb1, const __grid_constant__ CUtensorMap tc1,
                          GemmArgs g, int* dev_err) {
  pdl_trigger();  // the next slab's dz kernel may be scheduled as this grid's CTAs finish
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1k(smem_raw);
  uint8_t* sbox = smem + kPairStages * kPairStageBytes;  // two staging boxes, one per epilogue group
  __shared__ uint64_t full[kPairStages], empty[kPairStages], acc_full[2], acc_empty[2];
  __shared__ uint64_t item_full[4], item_empty[4], issued;
  __shared__ int item_q[4];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  volatile int* item_v = item_q;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int total = g.p[0].tiles + g.p[1].tiles;
  // item-queue consumers, all arriving on the leader's barrier: per CTA the
  // eight epilogue warps plus the MMA thread (leader) or the TMA thread (peer)
  constexpr int kItemConsumers = 2 * (1 + 8);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect-tx arrival (+ both CTAs' bytes)
      mbar_init(&empty[s], 1);  // the leader's commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // four epilogue warps of each CTA
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], kItemConsumers);
    }
    mbar_init(&issued, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == kHeadTma) {  // the same warp of both CTAs allocates the pair's TMEM
    tmem_alloc_pair(&tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  // launched as a programmatic dependent of the slab's dz kernel: the set-up
  // above overlapped its tail; dz and the tile counter are read only after it
  pdl_wait();
  const uint32_t item_empty0 = cluster_addr(&item_empty[0], 0);
  auto next_item = [&](int j, bool whole_warp) -> int {
    const int slot = j & 3;
    const bool ok = whole_warp ? mbar_wait_cluster_warp(&item_full[slot], (j >> 2) & 1, abort_v, dev_err)
                               : mbar_wait_cluster(&item_full[slot], (j >> 2) & 1, abort_v, dev_err);
    const int it = ok ? item_v[slot] : -1;
    if (whole_warp) __syncwarp();
    if (!whole_warp || lane == 0) mbar_arrive_cluster(item_empty0 + slot * 8);
    return it;
  };
  auto decode = [&](int it, int& p, int& m0, int& n0) {
    p = it < g.p[0].tiles ? 0 : 1;
    const int t = it - (p ? g.p[0].tiles : 0);
    m0 = (t / g.p[p].tiles_n) * kPairBM;
    n0 = (t % g.p[p].tiles_n) * kPairBN;
  };

  if (warp == kHeadTma) {
    if (lane == 0) {
      prefetch_tmap(&ta0);
      prefetch_tmap(&tb0);
      prefetch_tmap(&ta1);
      prefetch_tmap(&tb1);
      const uint32_t full0 = cluster_addr(&full[0], 0);  // the leader's stage barriers
      int it_stage = 0;
      int last_stage_it[kPairStages];
      for (int s = 0; s < kPairStages; ++s) last_stage_it[s] = -1;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        int it;
        if (leader) {
          // take the next tile and publish it in both CTAs' queues
          const int slot = j & 3;
          if (j >= 4 && !mbar_wait_cluster(&item_empty[slot], ((j >> 2) - 1) & 1, abort_v, dev_err)) break;
          it = atomicAdd(g.counter, 1);
          if (it >= total) it = -1;
          item_v[slot] = it;
          st_cluster_u32(cluster_addr(&item_q[slot], 1), (uint32_t)it);
          mbar_arrive(&item_full[slot]);
          mbar_arrive_cluster(cluster_addr(&item_full[slot], 1));  // release: the peer's copy is visible
        } else {
          it = next_item(j, false);
        }
        if (it < 0) break;
        int p, m0, n0;
        decode(it, p, m0, n0);
        const GemmProblem& P = g.p[p];
        const CUtensorMap* tA = p ? &ta1 : &ta0;
        const CUtensorMap* tB = p ? &tb1 : &tb0;
        const int ma = m0 + 128 * (int)rank, nb = n0 + 128 * (int)rank;  // this CTA's halves
        for (int kc = 0; kc < P.kchunks; ++kc, ++it_stage) {
          const int s = it_stage % kPairStages;
          if (it_stage >= kPairStages &&
              !mbar_wait_cluster(&empty[s], ((it_stage / kPairStages) - 1) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kPairStageBytes;
          uint8_t* sb = sa + kPairABytes;
          if (leader) mbar_expect_tx(&full[s], 2 * kPairStageBytes);  // both CTAs' halves
          const uint32_t fb = full0 + s * 8;
          const int k0 = kc * 64;
          if (P.a_mn) {  // [K][M] in memory: two 64-wide M chunks of 64 K rows
            tma_load_2d_pair(sa, tA, fb, ma, k0);
            tma_load_2d_pair(sa + kPairABytes / 2, tA, fb, ma + 64, k0);
          } else {  // [M][K]: one box of 128 rows x 64 K
            tma_load_2d_pair(sa, tA, fb, k0, ma);
          }
          // B is [K][N] (MN-major) in both problems: two 64-wide N chunks
          tma_load_2d_pair(sb, tB, fb, nb, k0);
          tma_load_2d_pair(sb + kPairBBytes / 2, tB, fb, nb + 64, k0);
          last_stage_it[s] = it_stage;
        }
      }
      if (*abort_v && leader)  // let copies in flight land (the leader's barriers count both CTAs')
        for (int s = 0; s < kPairStages; ++s)
          if (last_stage_it[s] >= 0) {
            volatile int quiet = 0;
            mbar_wait_cluster(&full[s], (last_stage_it[s] / kPairStages) & 1, &quiet, nullptr);
          }
    }
  } else if (warp == kHeadTma + 1) {
    if (lane == 0 && leader) {
      const uint32_t s0 = smem_u32(smem);
      const uint32_t empty0 = cluster_addr(&empty[0], 0), empty1 = cluster_addr(&empty[0], 1);
      const uint32_t accf0 = cluster_addr(&acc_full[0], 0), accf1 = cluster_addr(&acc_full[0], 1);
      int it_stage = 0;
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int it = next_item(j, false);
        if (it < 0) break;
        int p, m0, n0;
        decode(it, p, m0, n0);
        const GemmProblem& P = g.p[p];
        const uint32_t id = idesc_bf16_f32(kPairBM, kPairBN, P.a_mn, 1);
        const int buf = j & 1, use = j >> 1;
        if (use > 0 && !mbar_wait_cluster(&acc_empty[buf], (use - 1) & 1, abort_v, dev_err)) break;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * kPairBN;
        for (int kc = 0; kc < P.kchunks; ++kc, ++it_stage) {
          const int s = it_stage % kPairStages;
          if (!mbar_wait_cluster(&full[s], (it_stage / kPairStages) & 1, abort_v, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = s0 + s * kPairStageBytes, sb = sa + kPairABytes;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = P.a_mn ? desc_sw128(sa + k * 2048, kPairABytes / 2, 1024)
                                       : desc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = desc_sw128(sb + k * 2048, kPairBBytes / 2, 1024);
            mma_ss_pair(acc, ad, bd, id, (kc > 0 || k > 0));
          }
          mma_commit_pair(empty0 + s * 8);  // the stage is free again in both CTAs
          mma_commit_pair(empty1 + s * 8);
        }
        if (ok) {
          mma_commit_pair(accf0 + buf * 8);
          mma_commit_pair(accf1 + buf * 8);
        }
      }
      mma_commit_pair(cluster_addr(&issued, 0));  // settle before TMEM is freed
      volatile int quiet = 0;
      mbar_wait_cluster(&issued, 0, &quiet, dev_err);
    }
  } else {
    // epilogue group eg = warp / 4 takes the items j with j % 2 == eg; thread r
    // owns row r of this CTA's half of the tile
    const int eg = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    uint8_t* box = sbox + eg * kGemmBoxBytes;
    const bool issuer = (warp & 3) == 0 && lane == 0;
    const uint32_t acce0 = cluster_addr(&acc_empty[0], 0);
    for (int j = 0;; ++j) {
      const int it = next_item(j, true);
      if (it < 0) break;
      if ((j & 1) != eg) continue;
      int p, m0, n0;
      decode(it, p, m0, n0);
      const CUtensorMap* tC = p ? &tc1 : &tc0;
      const bool add = g.p[p].add != 0;
      const int use = j >> 1;
      const int mrow = m0 + 128 * (int)rank;
      if (!mbar_wait_cluster_warp(&acc_full[eg], use & 1, abort_v, dev_err)) break;
      tc_fence_after();
      const uint32_t acc = tmem_base + eg * kPairBN + lane_off;
#pragma unroll 1
      for (int c = 0; c < kPairBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(acc + 32 * c, v);
        if (c == kPairBN / 32 - 1) {  // the accumulator is read: the next tile may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(acce0 + eg * 8);
        }
        if (issuer) bulk_wait_group_read0();  // the previous box has been read by its TMA
        named_bar_sync(1 + eg, 128);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<uint4*>(box + r * 128 + ((u ^ (r & 7)) << 4)) =
              make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
        fence_proxy_async_smem();
        named_bar_sync(1 + eg, 128);
        if (issuer) {
          if (add)
            tma_reduce_add_2d(tC, box, n0 + 32 * c, mrow);
          else
            tma_store_2d(tC, box, n0 + 32 * c, mrow);
          bulk_commit_group();
        }
      }
    }
    if (issuer) bulk_wait_group0();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's last products (which read this CTA's shared memory) are done
  tc_fence_after();
  if (warp == kHeadTma) tmem_dealloc_pair(tmem_base, 512);
}

__global__ void f32_to_bf16_kernel(const float4* __restrict__ in, uint2* __restrict__ out, int64_t n4) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = in[i];
    out[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
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
    kern<<<dim3(tb, a.splits), kHeadThreads, kFwdSmem, st>>>(th, te, a, pm, pl, pz, device_error_word());  // tb even
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

template <int KIND>
// dependent: launch as a programmatic dependent of the previous kernel of the
// stream (every slab after the first; see head_dz_tc_kernel's epilogue).
int launch_dz_k(const CUtensorMap& th, const CUtensorMap& te, const CUtensorMap& tdz, const DzArgs& a, bool dependent,
                cudaStream_t st) {
  int dev = 0, sms = 0;
  ALGX_CUDA(cudaGetDevice(&dev));
  ALGX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const unsigned grid = 2u * (unsigned)std::max(1, std::min(a.items, sms / 2));  // persistent: one pair per 2 SMs
  auto run = [&](auto kern) -> int {
    ALGX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kDzSmem));
    if (dependent)
      ALGX_CUDA(launch_dependent(kern, grid, kHeadThreads, kDzSmem, st, th, te, tdz, a, device_error_word()));
    else
      kern<<<grid, kHeadThreads, kDzSmem, st>>>(th, te, tdz, a, device_error_word());
    ALGX_LAUNCHED("head_dz_tc launch");
    return ALGX_OK;
  };
  if (KIND == ALGX_HEAD_CE) return run(head_dz_tc_kernel<ALGX_HEAD_CE, 1>);
  switch (a.cfg.n) {
    case 2: return run(head_dz_tc_kernel<ALGX_HEAD_ALG_CE, 2>);
    case 4: return run(head_dz_tc_kernel<ALGX_HEAD_ALG_CE, 4>);
    case 8: return run(head_dz_tc_kernel<ALGX_HEAD_ALG_CE, 8>);
    case 16: return run(head_dz_tc_kernel<ALGX_HEAD_ALG_CE, 16>);
    default: return run(head_dz_tc_kernel<ALGX_HEAD_ALG_CE, 32>);
  }
}

int64_t slab_cols(int64_t V) {
  const int64_t vt = (V + kFwdNT - 1) / kFwdNT * kFwdNT;
  return std::min<int64_t>(kSlabCols, vt);
}

int launch_gemm_pair(const CUtensorMap (&maps)[6], const GemmArgs& a, cudaStream_t st) {
  int dev = 0, sms = 0;
  ALGX_CUDA(cudaGetDevice(&dev));
  ALGX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int total = a.p[0].tiles + a.p[1].tiles;
  const unsigned pairs = (unsigned)std::max(1, std::min(total, sms / 2));  // persistent: one pair per two SMs
  ALGX_CUDA(cudaFuncSetAttribute(head_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmem));
  // a programmatic dependent of the slab's dz kernel (it waits for it after its set-up)
  ALGX_CUDA(launch_dependent(head_gemm_pair_kernel, 2 * pairs, kGemmThreads, kPairSmem, st, maps[0], maps[1],
                             maps[2], maps[3], maps[4], maps[5], a, device_error_word()));
  ALGX_LAUNCHED("head_gemm_pair launch");
  return ALGX_OK;
}

}  // namespace
}  // namespace algx

using namespace algx;

extern "C" {

// Vocabulary splits of the forward: the grid is (256-token pairs) x splits
// CTA pairs of equal work, so the split count that minimises waves x (tiles
// per pair + about one tile of set-up) keeps the last wave of pairs full (3
// splits at N = 16384, V = 50304 left it 60% full; 8 fill it to ~97%).
int algx_head_fwd_splits(int64_t N, int64_t V) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t pairs = (N + 255) / 256, nt = (V + kFwdNT - 1) / kFwdNT, slots = std::max(1, sms / 2);
  int64_t best = 1, best_cost = INT64_MAX;
  for (int64_t s = 1; s <= std::min<int64_t>(nt, 64); ++s) {
    const int64_t cost = ((pairs * s + slots - 1) / slots) * ((nt + s - 1) / s + 1);  // + ~one tile of set-up per CTA
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return (int)best;
}

int algx_head_fwd(const algx_head_config* cfg, const void* h, const void* embed, const int32_t* targets,
                  float* part_m, float* part_l, float* part_zt, int64_t N, int64_t d, int64_t V, int64_t vocab_offset,
                  int32_t splits, int32_t dtype, void* stream) {
  if (int s = check_head(cfg, N, d, V, dtype)) return s;
  ALGX_REQUIRE(h && embed && targets && part_m && part_l && part_zt, "head_fwd: NULL pointer");
  ALGX_REQUIRE(splits >= 1 && splits <= 64, "head_fwd: splits must be in [1, 64]");
  CUtensorMap th, te;
  if (int s = make_tmap_2d(&th, h, ALGX_BF16, (uint64_t)d, (uint64_t)N, (uint64_t)d * 2, 64, 128, true)) return s;
  if (int s = make_tmap_2d(&te, embed, ALGX_BF16, (uint64_t)d, (uint64_t)V, (uint64_t)d * 2, 64, 128, true))
    return s;
  HeadArgs a{*cfg, targets, (int)N, (int)d, (int)V, (int)vocab_offset, splits};
  const int tb = 2 * (int)((N + 255) / 256);  // whole CTA pairs
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

size_t algx_head_bwd_workspace_size(int64_t N, int64_t d, int64_t V, int32_t dh_dtype) {
  if (N < 1 || d < 1 || V < 1) return 0;
  size_t bytes = (size_t)N * (size_t)slab_cols(V) * 2;               // dz slab, bf16
  if (dh_dtype == ALGX_BF16) bytes += (size_t)N * (size_t)d * 4;     // fp32 dh accumulator
  return bytes + 256;                                                // the GEMM tile counters (two)
}

int algx_head_bwd(const algx_head_config* cfg, const void* h, const void* embed, const int32_t* targets,
                  const float* stat, const float* scale, void* dh, int32_t dh_dtype, float* dembed, int64_t N,
                  int64_t d, int64_t V, int64_t vocab_offset, int32_t dtype, void* workspace, size_t workspace_bytes,
                  void* stream) {
  if (int s = check_head(cfg, N, d, V, dtype)) return s;
  ALGX_REQUIRE(h && embed && targets && stat && scale && dh && dembed, "head_bwd: NULL pointer");
  ALGX_REQUIRE(dh_dtype == ALGX_F32 || dh_dtype == ALGX_BF16, "head_bwd: dh dtype must be float32 or bfloat16");
  ALGX_REQUIRE(workspace && workspace_bytes >= algx_head_bwd_workspace_size(N, d, V, dh_dtype),
               "head_bwd: workspace too small (see algx_head_bwd_workspace_size)");
  const int64_t vs = slab_cols(V);
  CUtensorMap th, te;
  if (int s = make_tmap_2d(&th, h, ALGX_BF16, (uint64_t)d, (uint64_t)N, (uint64_t)d * 2, 64, 128, true)) return s;
  if (int s = make_tmap_2d(&te, embed, ALGX_BF16, (uint64_t)d, (uint64_t)V, (uint64_t)d * 2, 64, 128, true))
    return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __nv_bfloat16* dz = static_cast<__nv_bfloat16*>(workspace);
  float* dh_acc = dh_dtype == ALGX_F32 ? static_cast<float*>(dh)
                                       : reinterpret_cast<float*>(static_cast<char*>(workspace) + (size_t)N * vs * 2);
  // two GEMM tile counters, alternating by slab (each reset by its slab's dz kernel)
  int* counter = reinterpret_cast<int*>(static_cast<char*>(workspace) + algx_head_bwd_workspace_size(N, d, V, dh_dtype) -
                                        256);
  const int tbp = (int)((N + 255) / 256);  // 256-token blocks of the dz kernel's CTA pairs
  const int ntiles_total = (int)((V + kFwdNT - 1) / kFwdNT);
  const int tiles_n = (int)((d + kPairBN - 1) / kPairBN);
  // Slab s: dz kernel, then the GEMM that reads its dz, both programmatic
  // dependents of the kernel before them except the first dz kernel (a plain
  // launch: everything the chain reads besides dz is complete when it starts).
  // The dz buffer and the counters stay ordered by the kernels' own waits.
  for (int64_t c0 = 0, slab = 0; c0 < V; c0 += vs, ++slab) {
    const int64_t vc = std::min<int64_t>(vs, V - c0);  // valid columns of this slab
    DzArgs a{*cfg, targets, stat, scale, (int)N, (int)d, (int)V, (int)vocab_offset, (int)(c0 / kFwdNT), 0, 0};
    a.ntiles = std::min<int>((int)(vs / kFwdNT), ntiles_total - a.tile0);
    a.items = tbp * a.ntiles;
    a.gemm_counter = counter + (slab & 1);
    // the dz kernel's store map: the slab buffer, 128-row x 64-column boxes
    CUtensorMap tdz;
    int s = make_tmap_2d(&tdz, dz, ALGX_BF16, (uint64_t)vs, (uint64_t)N, (uint64_t)vs * 2, 64, 128, true);
    if (s) return s;
    s = cfg->kind == ALGX_HEAD_CE ? launch_dz_k<ALGX_HEAD_CE>(th, te, tdz, a, slab > 0, st)
                                  : launch_dz_k<ALGX_HEAD_ALG_CE>(th, te, tdz, a, slab > 0, st);
    if (s) return s;
    // problem 0: dE[c0 : c0 + vc] (vc x d) = dz^T . h; problem 1: dh (N x d) (+)= dz . E[c0 : c0 + vc]
    CUtensorMap maps[6];
    const __nv_bfloat16* eslab = static_cast<const __nv_bfloat16*>(embed) + (size_t)c0 * d;
    if ((s = make_tmap_2d(&maps[0], dz, ALGX_BF16, (uint64_t)vc, (uint64_t)N, (uint64_t)vs * 2, 64, 64, true))) return s;
    if ((s = make_tmap_2d(&maps[1], h, ALGX_BF16, (uint64_t)d, (uint64_t)N, (uint64_t)d * 2, 64, 64, true))) return s;
    if ((s = make_tmap_2d(&maps[2], dembed + (size_t)c0 * d, ALGX_F32, (uint64_t)d, (uint64_t)vc, (uint64_t)d * 4, 32,
                          128, true)))
      return s;
    if ((s = make_tmap_2d(&maps[3], dz, ALGX_BF16, (uint64_t)vc, (uint64_t)N, (uint64_t)vs * 2, 64, 128, true)))
      return s;
    if ((s = make_tmap_2d(&maps[4], eslab, ALGX_BF16, (uint64_t)d, (uint64_t)vc, (uint64_t)d * 2, 64, 64, true)))
      return s;
    if ((s = make_tmap_2d(&maps[5], dh_acc, ALGX_F32, (uint64_t)d, (uint64_t)N, (uint64_t)d * 4, 32, 128, true)))
      return s;
    GemmArgs ga;
    // 256-row tiles of CTA pairs; B (h for dE, E_slab for dh) is read MN-major in both problems
    ga.p[0] = GemmProblem{1, 1, 0, tiles_n, (int)((vc + kPairBM - 1) / kPairBM) * tiles_n, (int)((N + 63) / 64)};
    ga.p[1] = GemmProblem{0, 1, c0 > 0 ? 1 : 0, tiles_n, (int)((N + kPairBM - 1) / kPairBM) * tiles_n,
                          (int)((vc + 63) / 64)};
    ga.counter = a.gemm_counter;
    if ((s = launch_gemm_pair(maps, ga, st))) return s;
  }
  if (dh_dtype == ALGX_BF16) {
    const int64_t n4 = N * d / 4;
    f32_to_bf16_kernel<<<(unsigned)std::min<int64_t>((n4 + 255) / 256, 148 * 8), 256, 0, st>>>(
        reinterpret_cast<const float4*>(dh_acc), static_cast<uint2*>(dh), n4);
    ALGX_LAUNCHED("head dh rounding launch");
  }
  return ALGX_OK;
}

}  // extern "C"
