// XLA FFI handlers that let JAX call libalgx: the drop-in for the reference's
// Pallas kernels behind jax.ffi (kernels/flash.py:763, kernels/fused_head.py:260,
// kernels/qk_norm.py:62). Each handler unpacks the XLA buffers and forwards
// them to the C ABI of include/algx.h on XLA's CUDA stream; no handler
// allocates (workspaces arrive as extra result buffers that the Python shims
// size with the algx_*_workspace_size queries at trace time).
//
// Build (needs jaxlib for the header; see build.py next to this file):
//   g++ -O2 -std=c++17 -shared -fPIC -I<jax.ffi.include_dir()> -I<repo>/include \
//       algx_jax_ffi.cc -L<dir of libalgx.so> -lalgx -Wl,-rpath,<dir> -o libalgx_jax.so
#include <cuda_runtime_api.h>

#include <cstdint>
#include <string>

#include "algx.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error status_error(int status, const char* what) {
  if (status == ALGX_OK) return ffi::Error::Success();
  const ffi::ErrorCode code = status == ALGX_ERR_INVALID       ? ffi::ErrorCode::kInvalidArgument
                              : status == ALGX_ERR_UNSUPPORTED ? ffi::ErrorCode::kUnimplemented
                                                               : ffi::ErrorCode::kInternal;
  return ffi::Error(code, std::string(what) + ": " + algx_last_error());
}

// bf16 or f32 element type of an XLA buffer as the C ABI's dtype code (-1 otherwise).
int32_t dtype_of(const ffi::AnyBuffer& b) {
  switch (b.element_type()) {
    case ffi::DataType::BF16: return ALGX_BF16;
    case ffi::DataType::F32: return ALGX_F32;
    default: return -1;
  }
}

algx_attn_config attn_config(int32_t kind, int32_t mode, int32_t n, int32_t fast_rho, int32_t inv_stat,
                             int32_t has_sink, float clamp, float scale, float guard_qk, float guard_sink,
                             float guard_v) {
  algx_attn_config c;
  c.kind = kind;
  c.mode = mode;
  c.n = n;
  c.fast_rho = fast_rho;
  c.inv_stat = inv_stat;
  c.has_sink = has_sink;
  c.clamp = clamp;
  c.scale = scale;
  c.guard_qk = guard_qk;
  c.guard_sink = guard_sink;
  c.guard_v = guard_v;
  return c;
}

algx_head_config head_config(int32_t kind, int32_t n, float inv_c, float clamp, int32_t has_ignore,
                             int32_t ignore_index) {
  algx_head_config c;
  c.kind = kind;
  c.n = n;
  c.inv_c = inv_c;
  c.clamp = clamp;
  c.has_ignore = has_ignore;
  c.ignore_index = ignore_index;
  return c;
}

// ------------------------------------------------------------------ QK norm
ffi::Error QkNormFwd(cudaStream_t stream, ffi::AnyBuffer x, ffi::Buffer<ffi::F32> gain,
                     ffi::Result<ffi::AnyBuffer> y, float eps) {
  const int64_t rows = static_cast<int64_t>(x.element_count()) / 64;
  return status_error(algx_qknorm_fwd(x.untyped_data(), gain.typed_data(), y->untyped_data(), rows, 64,
                                      dtype_of(x), eps, stream),
                      "algx_qknorm_fwd");
}

ffi::Error QkNormBwd(cudaStream_t stream, ffi::AnyBuffer x, ffi::Buffer<ffi::F32> gain, ffi::AnyBuffer dy,
                     ffi::Result<ffi::AnyBuffer> dx, ffi::Result<ffi::Buffer<ffi::F32>> dgain,
                     ffi::Result<ffi::Buffer<ffi::U8>> workspace, float eps) {
  const int64_t rows = static_cast<int64_t>(x.element_count()) / 64;
  return status_error(algx_qknorm_bwd(x.untyped_data(), gain.typed_data(), dy.untyped_data(), dx->untyped_data(),
                                      dgain->typed_data(), rows, 64, dtype_of(x), eps, workspace->typed_data(),
                                      workspace->element_count(), stream),
                      "algx_qknorm_bwd");
}

// ---------------------------------------------------------------- attention
// Forward launch group: scale fold + guard maxima, then the causal forward.
// sink: (H,) fp32 in kernel units, or a zero-size buffer when has_sink == 0.
// o_precise: (B, H, T, D) fp32 on the guarded mode, zero-size otherwise.
ffi::Error AttnFwd(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v,
                   ffi::Buffer<ffi::F32> sink, ffi::Result<ffi::AnyBuffer> o, ffi::Result<ffi::Buffer<ffi::F32>> o_precise,
                   ffi::Result<ffi::Buffer<ffi::F32>> stat, ffi::Result<ffi::AnyBuffer> q_scaled,
                   ffi::Result<ffi::Buffer<ffi::F32>> guard, int32_t kind, int32_t mode, int32_t n, int32_t fast_rho,
                   int32_t inv_stat, int32_t has_sink, float clamp, float scale, float guard_qk, float guard_sink,
                   float guard_v) {
  const auto dims = q.dimensions();
  if (dims.size() != 4) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "q must be (B, H, T, D)");
  const int64_t B = dims[0], H = dims[1], T = dims[2], D = dims[3];
  const algx_attn_config cfg =
      attn_config(kind, mode, n, fast_rho, inv_stat, has_sink, clamp, scale, guard_qk, guard_sink, guard_v);
  const float* sk = has_sink ? sink.typed_data() : nullptr;
  const int32_t dt = dtype_of(q);
  if (int s = algx_attn_prepare(&cfg, q.untyped_data(), k.untyped_data(), v.untyped_data(), sk,
                                q_scaled->untyped_data(), guard->typed_data(), B, H, T, D, dt, stream))
    return status_error(s, "algx_attn_prepare");
  float* op = o_precise->element_count() ? o_precise->typed_data() : nullptr;
  return status_error(algx_attn_fwd(&cfg, q_scaled->untyped_data(), k.untyped_data(), v.untyped_data(), sk,
                                    guard->typed_data(), o->untyped_data(), op, stat->typed_data(), B, H, T, D, dt,
                                    stream),
                      "algx_attn_fwd");
}

// Backward launch group; dq is d/dq of the unscaled q (the scale fold applied).
ffi::Error AttnBwd(cudaStream_t stream, ffi::AnyBuffer q_scaled, ffi::AnyBuffer k, ffi::AnyBuffer v,
                   ffi::Buffer<ffi::F32> sink, ffi::Buffer<ffi::F32> guard, ffi::AnyBuffer o,
                   ffi::Buffer<ffi::F32> o_precise, ffi::Buffer<ffi::F32> stat, ffi::AnyBuffer dout,
                   ffi::Result<ffi::AnyBuffer> dq, ffi::Result<ffi::AnyBuffer> dk, ffi::Result<ffi::AnyBuffer> dv,
                   ffi::Result<ffi::Buffer<ffi::F32>> dsink, ffi::Result<ffi::Buffer<ffi::U8>> workspace, int32_t kind,
                   int32_t mode, int32_t n, int32_t fast_rho, int32_t inv_stat, int32_t has_sink, float clamp,
                   float scale, float guard_qk, float guard_sink, float guard_v) {
  const auto dims = q_scaled.dimensions();
  if (dims.size() != 4) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "q must be (B, H, T, D)");
  const int64_t B = dims[0], H = dims[1], T = dims[2], D = dims[3];
  const algx_attn_config cfg =
      attn_config(kind, mode, n, fast_rho, inv_stat, has_sink, clamp, scale, guard_qk, guard_sink, guard_v);
  const float* sk = has_sink ? sink.typed_data() : nullptr;
  const float* op = o_precise.element_count() ? o_precise.typed_data() : nullptr;
  float* ds = has_sink ? dsink->typed_data() : nullptr;
  return status_error(algx_attn_bwd(&cfg, q_scaled.untyped_data(), k.untyped_data(), v.untyped_data(), sk,
                                    guard.typed_data(), o.untyped_data(), op, stat.typed_data(), dout.untyped_data(),
                                    dq->untyped_data(), dk->untyped_data(), dv->untyped_data(), ds, B, H, T, D,
                                    dtype_of(q_scaled), workspace->typed_data(), workspace->element_count(), stream),
                      "algx_attn_bwd");
}

// ---------------------------------------------------------------- fused head
// Forward: per-split partials, their combination and the objective; partials
// (3, splits, N) and mlz (3, N) are scratch results. objective and count are
// (1,) fp32 device scalars; stat and telemetry (N,).
ffi::Error HeadFwd(cudaStream_t stream, ffi::AnyBuffer h, ffi::AnyBuffer embed, ffi::Buffer<ffi::S32> targets,
                   ffi::Result<ffi::Buffer<ffi::F32>> objective, ffi::Result<ffi::Buffer<ffi::F32>> telemetry,
                   ffi::Result<ffi::Buffer<ffi::F32>> stat, ffi::Result<ffi::Buffer<ffi::F32>> count,
                   ffi::Result<ffi::Buffer<ffi::F32>> partials, ffi::Result<ffi::Buffer<ffi::F32>> mlz, int32_t kind,
                   int32_t n, float inv_c, float clamp, int32_t has_ignore, int32_t ignore_index) {
  const auto hd = h.dimensions();
  const auto ed = embed.dimensions();
  if (hd.size() != 2 || ed.size() != 2) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "h (N, d), embed (V, d)");
  const int64_t N = hd[0], d = hd[1], V = ed[0];
  const algx_head_config cfg = head_config(kind, n, inv_c, clamp, has_ignore, ignore_index);
  const int32_t splits = algx_head_fwd_splits(N, V);
  if ((int64_t)partials->element_count() < 3 * (int64_t)splits * N)
    return ffi::Error(ffi::ErrorCode::kInvalidArgument, "head partials buffer too small");
  float* pm = partials->typed_data();
  float* pl = pm + (size_t)splits * N;
  float* pz = pl + (size_t)splits * N;
  if (int s = algx_head_fwd(&cfg, h.untyped_data(), embed.untyped_data(), targets.typed_data(), pm, pl, pz, N, d, V,
                            0, splits, dtype_of(h), stream))
    return status_error(s, "algx_head_fwd");
  float* m = mlz->typed_data();
  if (int s = algx_head_reduce(&cfg, pm, pl, pz, splits, N, m, m + N, m + 2 * N, stream))
    return status_error(s, "algx_head_reduce");
  return status_error(algx_head_finalize(&cfg, targets.typed_data(), m, m + N, m + 2 * N, N, V, stat->typed_data(),
                                         telemetry->typed_data(), objective->typed_data(), count->typed_data(),
                                         stream),
                      "algx_head_finalize");
}

// Backward: dh (h's dtype) and dembed (fp32); scale = g * slope / count is a
// (1,) fp32 device scalar computed by the shim.
ffi::Error HeadBwd(cudaStream_t stream, ffi::AnyBuffer h, ffi::AnyBuffer embed, ffi::Buffer<ffi::S32> targets,
                   ffi::Buffer<ffi::F32> stat, ffi::Buffer<ffi::F32> scale, ffi::Result<ffi::AnyBuffer> dh,
                   ffi::Result<ffi::Buffer<ffi::F32>> dembed, ffi::Result<ffi::Buffer<ffi::U8>> workspace, int32_t kind,
                   int32_t n, float inv_c, float clamp, int32_t has_ignore, int32_t ignore_index) {
  const auto hd = h.dimensions();
  const auto ed = embed.dimensions();
  const int64_t N = hd[0], d = hd[1], V = ed[0];
  const algx_head_config cfg = head_config(kind, n, inv_c, clamp, has_ignore, ignore_index);
  return status_error(algx_head_bwd(&cfg, h.untyped_data(), embed.untyped_data(), targets.typed_data(),
                                    stat.typed_data(), scale.typed_data(), dh->untyped_data(), dtype_of(*dh),
                                    dembed->typed_data(), N, d, V, 0, dtype_of(h), workspace->typed_data(),
                                    workspace->element_count(), stream),
                      "algx_head_bwd");
}

}  // namespace

#define ALGX_ATTN_ATTRS                                                                                      \
  .Attr<int32_t>("kind").Attr<int32_t>("mode").Attr<int32_t>("n").Attr<int32_t>("fast_rho")                  \
      .Attr<int32_t>("inv_stat").Attr<int32_t>("has_sink").Attr<float>("clamp").Attr<float>("scale")         \
      .Attr<float>("guard_qk").Attr<float>("guard_sink").Attr<float>("guard_v")
#define ALGX_HEAD_ATTRS                                                                                      \
  .Attr<int32_t>("kind").Attr<int32_t>("n").Attr<float>("inv_c").Attr<float>("clamp")                       \
      .Attr<int32_t>("has_ignore").Attr<int32_t>("ignore_index")

XLA_FFI_DEFINE_HANDLER_SYMBOL(AlgxQkNormFwd, QkNormFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Attr<float>("eps"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(AlgxQkNormBwd, QkNormBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<float>("eps"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(AlgxAttnFwd, AttnFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>() ALGX_ATTN_ATTRS);

XLA_FFI_DEFINE_HANDLER_SYMBOL(AlgxAttnBwd, AttnBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>() ALGX_ATTN_ATTRS);

XLA_FFI_DEFINE_HANDLER_SYMBOL(AlgxHeadFwd, HeadFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::F32>>() ALGX_HEAD_ATTRS);

XLA_FFI_DEFINE_HANDLER_SYMBOL(AlgxHeadBwd, HeadBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::AnyBuffer>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::AnyBuffer>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Ret<ffi::Buffer<ffi::U8>>() ALGX_HEAD_ATTRS);
