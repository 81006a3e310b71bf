// Attention variant resolution shared by the generic and tcgen05 kernels.
#pragma once

#include "algx_common.cuh"

namespace algx {

// Accumulation branch actually executed.
enum Branch : int { BR_UNSHIFTED = 0, BR_SHIFTED = 1, BR_SOFTMAX = 2 };

struct Eff {
  int branch;     // Branch
  bool clip;      // unshifted with the upper score clamp (explicit shift=False)
  bool fast;      // fast rho for score weights (flash.py:83-88)
  bool inv_stat;  // unshifted statistic 1/Z instead of Z^(-1/n)
  bool precise;   // guarded high branch: keep the unrounded output (flash.py:851-852)
};

// Variant of kernels/flash.py:732-760, with the range-guard decision of
// flash.py:834-856 taken on the device from the maxima algx_attn_prepare
// wrote: guard[0] = max||q_s||^2, [1] = max||k||^2, [2] = max|v|, [3] = max|sink|.
// A NaN maximum fails every comparison and selects the shifted branch, as
// the reference's lax.cond does.
__host__ __device__ inline Eff resolve_variant(const algx_attn_config& c, const float* guard) {
  Eff e{BR_UNSHIFTED, false, c.fast_rho != 0, c.inv_stat != 0, false};
  if (c.kind == ALGX_ATTN_SOFTMAX) {
    e.branch = BR_SOFTMAX;
    e.fast = false;
    e.inv_stat = false;
    return e;
  }
  if (c.mode == ALGX_MODE_CLIPPED) {
    e.clip = true;
    return e;
  }
  if (c.mode == ALGX_MODE_SHIFTED) {
    e.branch = BR_SHIFTED;
    e.inv_stat = false;
    return e;
  }
  bool ok = guard[0] * guard[1] <= c.guard_qk;
  if (c.has_sink) ok = ok && guard[3] <= c.guard_sink;
  ok = ok && guard[2] <= c.guard_v;
  if (ok) {
    e.inv_stat = true;  // low = var._replace(shift=False, inv_stat=True, bounded_scores=True)
  } else {
    e.branch = BR_SHIFTED;  // high: shift, exact rho, root statistic, precise output
    e.fast = false;
    e.inv_stat = false;
    e.precise = true;
  }
  return e;
}

// Whether the tcgen05 backward (when it was launched: bf16, D = 64, T % 128
// == 0, asinh fast path) produced this branch's gradients in its fp32 dQ
// accumulator: the unshifted branch always, the shifted one under the range
// guard (kernels/flash.py:834-856), where both instantiations are launched.
__host__ __device__ inline bool tc_bwd_covers(const algx_attn_config& c, const Eff& e) {
  return e.branch == BR_UNSHIFTED || (e.branch == BR_SHIFTED && c.mode == ALGX_MODE_GUARDED);
}

}  // namespace algx
