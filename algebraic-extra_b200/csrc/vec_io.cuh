// 128-bit row I/O helpers for D = 64 rows (bf16: 8 threads per row, fp32: 16).
#pragma once

#include "algx_common.cuh"

namespace algx {

constexpr int kRowDim = 64;

template <typename T> struct Vec {
  static constexpr int N = 16 / sizeof(T);   // elements per 16-byte chunk
  static constexpr int TPR = kRowDim / N;       // threads per row
  static constexpr int RPW = 32 / TPR;       // rows per warp per pass
};

template <typename T>
__device__ __forceinline__ void unpack(const uint4& raw, float (&v)[Vec<T>::N]) {
  if constexpr (sizeof(T) == 4) {
    v[0] = __uint_as_float(raw.x); v[1] = __uint_as_float(raw.y);
    v[2] = __uint_as_float(raw.z); v[3] = __uint_as_float(raw.w);
  } else {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float (&v)[Vec<T>::N]) {
  uint4 raw;
  if constexpr (sizeof(T) == 4) {
    raw.x = __float_as_uint(v[0]); raw.y = __float_as_uint(v[1]);
    raw.z = __float_as_uint(v[2]); raw.w = __float_as_uint(v[3]);
  } else {
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  }
  return raw;
}

template <int TPR>
__device__ __forceinline__ float row_sum(float s) {
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }

}  // namespace algx
