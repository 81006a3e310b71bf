// Library-wide C ABI pieces: error strings, version, the per-device error
// word, and the TMA tensor-map encoder (resolved from the driver at runtime,
// so the library does not link libcuda directly).
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <string>

#include "algx_common.cuh"
#include "tmap.h"

namespace algx {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int check_cuda(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return ALGX_OK;
  g_last_error = std::string(what) + ": " + cudaGetErrorString(err);
  return ALGX_ERR_CUDA;
}

// One device int per device, allocated on first use (before any capture).
static std::mutex g_err_mu;
static int* g_err_word[64] = {nullptr};

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_err_mu);
  if (!g_err_word[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_err_word[dev] = p;
  }
  return g_err_word[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int make_tmap_2d(CUtensorMap* map, const void* base, int32_t dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(ALGX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(ALGX_ERR_INVALID, "TMA base not 16-byte aligned");
  if (row_stride_bytes % 16 != 0) return fail(ALGX_ERR_INVALID, "TMA row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType t = dtype == ALGX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = g_encode(map, t, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ALGX_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return ALGX_OK;
}

}  // namespace algx

extern "C" {

const char* algx_last_error(void) { return algx::g_last_error.c_str(); }

int algx_version(void) { return 100; }

uint64_t algx_launch_count(void) { return algx::g_launches.load(std::memory_order_relaxed); }

int algx_device_error(int32_t* code) {
  if (!code) return algx::fail(ALGX_ERR_INVALID, "code is NULL");
  int* w = algx::device_error_word();
  if (!w) return algx::fail(ALGX_ERR_CUDA, "device error word unavailable");
  ALGX_CUDA(cudaDeviceSynchronize());
  int v = 0;
  ALGX_CUDA(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  ALGX_CUDA(cudaMemset(w, 0, sizeof(int)));
  *code = v;
  return ALGX_OK;
}

}  // extern "C"
