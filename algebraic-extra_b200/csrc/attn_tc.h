// tcgen05 fast path of the attention (bf16, D = 64, T % 128 == 0, asinh;
// the unshifted branch, and under the range guard the shifted one too). Each
// launcher sets *launched when it took the call; the generic kernels then
// skip the branches it covers.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "algx.h"

namespace algx {

// o_prec: the fp32 output the guarded mode's shifted branch also writes
// (may be null outside the guarded mode).
int tc_attn_fwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v,
                const float* sink, const float* guard, void* o, float* o_prec, float* stat, int64_t B, int64_t H,
                int64_t T, int32_t dtype, cudaStream_t st, bool* launched);

// With finish_dq false the fp32 dQ accumulator (the first B*H*T*64 floats of
// the workspace, unscaled) is left for the caller instead of being rounded
// into dq.
// pre_zeroed: the caller has already zeroed the accumulator and the 256-byte
// counter area that follows it (the di pass does), so no memset is issued.
int tc_attn_bwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v,
                const void* dout, const float* stat, const float* di, const float* guard, void* dq, void* dk,
                void* dv, void* workspace, int64_t B, int64_t H, int64_t T, int32_t dtype, cudaStream_t st,
                bool finish_dq, bool pre_zeroed, bool* launched);

// Whether tc_attn_bwd takes a call with this configuration.
bool tc_attn_bwd_eligible(const algx_attn_config& cfg, int64_t T, int32_t dtype);

// Byte offset, within the fast-path workspace, of 64 spare bytes that the
// launch zeroes along with the dQ accumulator.
size_t tc_attn_bwd_spare_offset(int64_t B, int64_t H, int64_t T, int64_t D);

size_t tc_attn_bwd_workspace(int64_t B, int64_t H, int64_t T, int64_t D);

}  // namespace algx
