// Shared host/device helpers for libalgx: status codes, dtype access and the
// reference's scalar maths (rho, integer powers, inverse roots).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "algx.h"

namespace algx {

// ---------------------------------------------------------------- host side
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_cuda(cudaError_t err, const char* what);
void count_launches(int n);

#define ALGX_REQUIRE(cond, msg) \
  do { if (!(cond)) return ::algx::fail(ALGX_ERR_INVALID, (msg)); } while (0)
#define ALGX_CUDA(call) \
  do { int _s = ::algx::check_cuda((call), #call); if (_s) return _s; } while (0)
#define ALGX_LAUNCHED(what) \
  do { ::algx::count_launches(1); int _s = ::algx::check_cuda(cudaGetLastError(), what); if (_s) return _s; } while (0)

// Device-side error word. A bounded wait that gives up ORs a code in here
// instead of spinning forever; algx_device_error() reads and clears it.
enum DeviceError : int {
  DEV_ERR_MBAR_TIMEOUT = 1,
  DEV_ERR_TMEM_ALLOC = 2,
  DEV_ERR_BAD_LABEL = 4,
};

// Programmatic dependent launch: a kernel launched with launch_dependent() may
// start while the previous kernel of the stream is still running, once every
// block of that kernel has called pdl_trigger() (or exited); it must call
// pdl_wait() before it reads the previous kernel's results or exits, so that
// later work in the stream stays ordered after both.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- device side
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
// Round a float32 value through the I/O type (identity for float32).
template <typename T> __device__ __forceinline__ float round_io(float x) {
  return to_f32(from_f32<T>(x));
}

// x^n by binary exponentiation (algebraic.py:38-51).
__device__ __forceinline__ float ipow(float x, int n) {
  float out = 1.f;
  bool first = true;
  float base = x;
  while (n) {
    if (n & 1) { out = first ? base : out * base; first = false; }
    n >>= 1;
    if (n) base = base * base;
  }
  return out;
}
template <int N> __device__ __forceinline__ float ipow_t(float x) {
  if constexpr (N == 1) return x;
  else if constexpr ((N & 1) == 0) { float h = ipow_t<N / 2>(x); return h * h; }
  else return x * ipow_t<N - 1>(x);
}

// 1/sqrt(x) on the MUFU pipe, flushing denormals (the arguments here are
// 1 + x^2 >= 1 or positive row sums, never denormal).
__device__ __forceinline__ float rsqrt_fast(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 1/x on the MUFU pipe (approximate reciprocal, flushing denormals; the
// arguments here are |x| + sqrt(1 + x^2) >= 1).
__device__ __forceinline__ float rcp_fast(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// rho(x) = x + sqrt(1+x^2): fast form (kernels/flash.py:83-88) and stable
// form with the reciprocal for x < 0 (kernels/flash.py:76-80). Both return
// r = 1/sqrt(1+x^2) through the out-parameter.
__device__ __forceinline__ float rho_fast(float x, float& r) {
  float rad = fmaf(x, x, 1.f);
  r = rsqrtf(rad);
  return fmaf(rad, r, x);
}
__device__ __forceinline__ float rho_exact(float x, float& r) {
  float rad = fmaf(x, x, 1.f);
  r = rsqrtf(rad);
  float t = fabsf(x) + rad * r;
  return x >= 0.f ? t : 1.f / t;
}
__device__ __forceinline__ float rho_sel(float x, bool fast, float& r) {
  return fast ? rho_fast(x, r) : rho_exact(x, r);
}
// l^(-1/n), n a power of two (kernels/flash.py:107-114).
__device__ __forceinline__ float inv_root(float l, int n) {
  float y = rsqrtf(l);
  for (int k = n / 2; k > 1; k /= 2) y = y * rsqrtf(y);
  return y;
}

// Packed FP32 pairs (sm_100 f32x2 arithmetic): two lanes of work per
// instruction on the FMA pipe.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
template <int N> __device__ __forceinline__ float2 ipow2_t(float2 x) {
  if constexpr (N == 1) return x;
  else if constexpr ((N & 1) == 0) { float2 h = ipow2_t<N / 2>(x); return mul2(h, h); }
  else return mul2(x, ipow2_t<N - 1>(x));
}

// Reinterpretation helpers for order-preserving float max via integer atomics
// on non-negative values.
__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
}

}  // namespace algx
