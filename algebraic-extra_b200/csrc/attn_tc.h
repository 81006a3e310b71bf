// tcgen05 fast path of the attention (bf16, D = 64, T % 128 == 0, asinh
// unshifted branch). Each launcher sets *launched when it took the call;
// the generic kernels then skip the unshifted branch.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "algx.h"

namespace algx {

int tc_attn_fwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v,
                const float* sink, const float* guard, void* o, float* stat, int64_t B, int64_t H, int64_t T,
                int32_t dtype, cudaStream_t st, bool* launched);

int tc_attn_bwd(const algx_attn_config& cfg, const void* q_scaled, const void* k, const void* v,
                const void* dout, const float* stat, const float* di, const float* guard, void* dq, void* dk,
                void* dv, void* workspace, int64_t B, int64_t H, int64_t T, int32_t dtype, cudaStream_t st,
                bool* launched);

size_t tc_attn_bwd_workspace(int64_t B, int64_t H, int64_t T, int64_t D);

}  // namespace algx
