/*
 * libalgx: C ABI of the B200 (sm_100a) kernels for the Algebraic Transformer
 * hot path (asinh-power flash attention, fused LM head, QK RMS norm).
 *
 * Conventions for every entry point:
 *   - pointers are device pointers unless stated; tensors are contiguous,
 *     row-major; attention tensors are (B, H, T, D), D = 64;
 *   - `stream` is a cudaStream_t (NULL = legacy default stream);
 *   - the library never allocates device memory on a call path: the caller
 *     passes outputs and any workspace (sized by the *_workspace_size query);
 *   - calls are stream-ordered and never synchronize the host;
 *   - the return value is an algx status; on failure algx_last_error()
 *     returns a message for the calling thread.
 *
 * Each declaration names the reference function it replaces
 * (paths relative to the reference project, tasmaikeni13/algebraic-extra).
 */
#ifndef ALGX_H_
#define ALGX_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ALGX_API __attribute__((visibility("default")))
#else
#define ALGX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum { ALGX_OK = 0, ALGX_ERR_INVALID = 1, ALGX_ERR_UNSUPPORTED = 2, ALGX_ERR_CUDA = 3 };
enum { ALGX_F32 = 0, ALGX_BF16 = 1 };
enum { ALGX_ATTN_ASINH = 0, ALGX_ATTN_SOFTMAX = 1 };
/* asinh accumulation strategy (kernels/flash.py:9-22):
 *   CLIPPED  unshifted, scores clamped above at `clamp` (explicit shift=False);
 *   SHIFTED  running maximum with rho(-m) shifts (explicit shift=True);
 *   GUARDED  range_guard=True: the device picks unshifted-unclamped when the
 *            Cauchy-Schwarz guard passes, else shifted with exact rho. */
enum { ALGX_MODE_CLIPPED = 0, ALGX_MODE_SHIFTED = 1, ALGX_MODE_GUARDED = 2 };
enum { ALGX_HEAD_CE = 0, ALGX_HEAD_ALG_CE = 1 };

/* Message of the last failed call on this thread. Library plumbing:
 * no counterpart in the reference (its kernels raise Python exceptions). */
ALGX_API const char* algx_last_error(void);
/* Library version (major*10000 + minor*100 + patch).
 * No counterpart in the reference. */
ALGX_API int algx_version(void);
/* Number of kernels this process launched through libalgx so far.
 * No counterpart in the reference. */
ALGX_API uint64_t algx_launch_count(void);
/* Reads and clears the device error word of the current device (bounded
 * waits that gave up set it). Synchronizes the device. No counterpart in the
 * reference (a Pallas kernel has no bounded device-side waits). */
ALGX_API int algx_device_error(int32_t* code);

/* ------------------------------------------------------------------ QK norm */

/* y = rms_norm(x) * gain over rows of `dim` (= 64) elements.
 * Replaces kernels/qk_norm.py:62-76 `qk_rms_norm` forward (algebraic.py:76-83). */
ALGX_API int algx_qknorm_fwd(const void* x, const float* gain, void* y, int64_t rows, int64_t dim,
                    int32_t dtype, float eps, void* stream);

/* Bytes of workspace algx_qknorm_bwd needs. No counterpart in the reference: XLA sizes the Pallas kernels' scratch itself. */
ALGX_API size_t algx_qknorm_bwd_workspace_size(int64_t rows, int64_t dim);

/* dx and dgain of the QK norm. Replaces kernels/qk_norm.py:39-55 `_norm_bwd`
 * (dx by the AD formula of rms_norm, dgain = sum_rows dy * x * tau). */
ALGX_API int algx_qknorm_bwd(const void* x, const float* gain, const void* dy, void* dx, float* dgain,
                    int64_t rows, int64_t dim, int32_t dtype, float eps, void* workspace,
                    size_t workspace_bytes, void* stream);

/* QK-norm backward that allocates nothing, for callers that cannot call
 * cudaMalloc (a host framework that owns all device memory, code running
 * while a pool allocator is locked, or a foreign-function layer with no
 * workspace channel). No counterpart in the reference.
 * Same arguments and results as algx_qknorm_bwd minus the workspace: the
 * per-CTA dgain partials live in a library-owned static device array of
 * 256 x 64 fp32 (64 KiB per device, kept until the process exits).
 * Limits: rows <= 2147483647 (larger counts return ALGX_ERR_INVALID).
 * The first call on each device looks up the array's device address; make
 * that first call before any stream capture. Every call shares the array, so
 * calls that overlap on the GPU (other streams, other threads) race; serialise
 * them on one stream. */
ALGX_API int algx_qknorm_bwd_noalloc(const void* x, const float* gain, const void* dy, void* dx, float* dgain,
                                     int64_t rows, int64_t dim, int32_t dtype, float eps, void* stream);

/* ---------------------------------------------------------------- attention */

/* Resolved variant of kernels/flash.py:732-760 plus the wrapper's constants. */
typedef struct algx_attn_config {
  int32_t kind;     /* ALGX_ATTN_ASINH or ALGX_ATTN_SOFTMAX */
  int32_t mode;     /* ALGX_MODE_* (asinh only) */
  int32_t n;        /* weight power, a power of two >= 2 */
  int32_t fast_rho; /* 1: rho(x) = x + rad*rsqrt(rad) (flash.py:83-88) */
  int32_t inv_stat; /* unshifted row statistic: 1 -> 1/Z, 0 -> Z^(-1/n) */
  int32_t has_sink; /* sink logit present (kernel units, shape (H,)) */
  float clamp;      /* make_variant clamp, kernel units (flash.py:747-748) */
  float scale;      /* 1/(sqrt(D)*unit), folded into q (flash.py:823-833) */
  float guard_qk;   /* (bound/1.01)^2 (flash.py:840-843) */
  float guard_sink; /* bound/1.01 (flash.py:844-845) */
  float guard_v;    /* vmax (flash.py:848-849) */
} algx_attn_config;

/* q_scaled = (q*scale) rounded to the I/O dtype, and the range-guard maxima
 * guard[0] = max ||q_scaled||^2, guard[1] = max ||k||^2, guard[2] = max |v|,
 * guard[3] = max |sink| (guard: 4 device floats, overwritten).
 * Replaces the XLA glue of kernels/flash.py:823-849. */
ALGX_API int algx_attn_prepare(const algx_attn_config* cfg, const void* q, const void* k, const void* v,
                      const float* sink, void* q_scaled, float* guard, int64_t B, int64_t H,
                      int64_t T, int64_t D, int32_t dtype, void* stream);

/* Fused attention prologue: the QK RMS norm of q and k followed by
 * algx_attn_prepare, in one pass. k_norm = round(rmsnorm(k) * gain_k) and
 * q_scaled = round(round(rmsnorm(q) * gain_q) * scale) are bit-identical to
 * algx_qknorm_fwd on q and k followed by algx_attn_prepare; guard as there.
 * Replaces the model's qk-norm -> rotary -> flash_attention prologue
 * (model.py:170-174, qk_norm.py:29-43, algebraic.py:172-179,
 * flash.py:823-849). rope_cos, rope_sin: NULL (no rotary) or (rope_rows >= T,
 * 32) fp32 tables, row t for position t (RoPE, standard.py:16-21, or Cayley,
 * algebraic.py:124-169); the rotation runs between the norm and the scale
 * fold, rounded to the I/O dtype once. */
ALGX_API int algx_qknorm_attn_prepare(const algx_attn_config* cfg, const void* q, const void* k,
                                      const void* v, const float* gain_q, const float* gain_k,
                                      const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                                      const float* sink, void* q_scaled, void* k_norm, float* guard,
                                      int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype, float eps,
                                      void* stream);

/* Causal forward: o (I/O dtype), stat (B,H,T) fp32, and on the shifted
 * guard fallback the unrounded output o_precise (B,H,T,D) fp32 (nullable when
 * cfg->mode != GUARDED). Replaces kernels/flash.py:189-326 `_forward` and
 * kernels/head_resident.py:24-155 `forward`. */
ALGX_API int algx_attn_fwd(const algx_attn_config* cfg, const void* q_scaled, const void* k, const void* v,
                  const float* sink, const float* guard, void* o, float* o_precise, float* stat,
                  int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype, void* stream);

/* Bytes of workspace algx_attn_bwd needs. No counterpart in the reference: XLA sizes the Pallas kernels' scratch itself. */
ALGX_API size_t algx_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D);

/* Causal backward: dq (with the scale fold applied, i.e. d/dq of the
 * unscaled q), dk, dv and, when cfg->has_sink, dsink (H,) fp32 in kernel
 * units. Replaces kernels/flash.py:630-642 `_backward` (+ :435-627,
 * head_resident.py:95-176) and the sink VJP of flash.py:694-726. */
ALGX_API int algx_attn_bwd(const algx_attn_config* cfg, const void* q_scaled, const void* k, const void* v,
                  const float* sink, const float* guard, const void* o, const float* o_precise,
                  const float* stat, const void* dout, void* dq, void* dk, void* dv, float* dsink,
                  int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Bytes of workspace algx_qknorm_attn_bwd needs. No counterpart in the reference: XLA sizes the Pallas kernels' scratch itself. */
ALGX_API size_t algx_qknorm_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D);

/* Backward of attention over QK-normed inputs, the counterpart of
 * algx_qknorm_attn_prepare: the attention backward of algx_attn_bwd on
 * (q_scaled, k_norm) followed by the QK RMS norm backward of q and k
 * (kernels/qk_norm.py:45-56) in one launch group. dq, dk receive d/dq and
 * d/dk of the raw (pre-norm) q, k (through the inverse rotation when
 * rope_cos, rope_sin are given, as in algx_qknorm_attn_prepare); dgain_q,
 * dgain_k (64,) fp32 the gain
 * gradients; dv and dsink as algx_attn_bwd. dk equals, bit for bit,
 * algx_attn_bwd followed by algx_qknorm_bwd, and so does dq up to the order
 * of the fast path's dQ reduce-adds (which varies between any two calls);
 * dgain differs only by the order of its fp32 sums. Replaces the VJP of the model's qk-norm ->
 * flash_attention prologue (model.py:170-174: qk_norm.py:45-56 after
 * flash.py:630-642). */
ALGX_API int algx_qknorm_attn_bwd(const algx_attn_config* cfg, const void* q, const void* k, const float* gain_q,
                  const float* gain_k, const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                  const void* q_scaled, const void* k_norm, const void* v,
                  const float* sink, const float* guard, const void* o, const float* o_precise,
                  const float* stat, const void* dout, void* dq, void* dk, void* dv, float* dgain_q,
                  float* dgain_k, float* dsink, int64_t B, int64_t H, int64_t T, int64_t D, int32_t dtype,
                  float eps, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------- fused head */

/* kernels/fused_head.py:260-275 (+ the ignore_index extension). */
typedef struct algx_head_config {
  int32_t kind;         /* ALGX_HEAD_CE or ALGX_HEAD_ALG_CE */
  int32_t n;            /* alg_ce power (2..32, power of two) */
  float inv_c;          /* 1/c */
  float clamp;          /* alg_ce kernel-argument clamp X = 0.25*(1e38/V)^(1/n) (fused_head.py:273) */
  int32_t has_ignore;   /* 1: rows with target == ignore_index leave loss, gradients and mean */
  int32_t ignore_index;
} algx_head_config;

/* Vocabulary splits algx_head_fwd uses for N tokens over V local rows. */
ALGX_API int algx_head_fwd_splits(int64_t N, int64_t V);

/* Forward partial statistics per (split, token): running max m, sum l and
 * target logit zt over this rank's V vocabulary rows (global row index =
 * local + vocab_offset). h (N, d) and embed (V, d) are bf16, d % 64 == 0.
 * part_* are (splits, N) fp32. Replaces kernels/fused_head.py:72-117
 * `_fwd_kernel` / `_forward` without materialising the logits. */
ALGX_API int algx_head_fwd(const algx_head_config* cfg, const void* h, const void* embed,
                           const int32_t* targets, float* part_m, float* part_l, float* part_zt,
                           int64_t N, int64_t d, int64_t V, int64_t vocab_offset, int32_t splits,
                           int32_t dtype, void* stream);

/* Combine split partials into one (m, l, zt) per token (max and rescaled
 * sum for ce; plain sums for alg_ce). Part of fused_head.py:174-191. */
ALGX_API int algx_head_reduce(const algx_head_config* cfg, const float* part_m, const float* part_l,
                              const float* part_zt, int32_t splits, int64_t N, float* m, float* l,
                              float* zt, void* stream);

/* stat (lse or l^(-1/n)), telemetry (nll or target probability), objective
 * (device scalar) and the loss row count (device scalar). Replaces
 * kernels/fused_head.py:219-229 `_telemetry`. Labels outside [0, V_total)
 * other than ignore_index raise the device error word when has_ignore. */
ALGX_API int algx_head_finalize(const algx_head_config* cfg, const int32_t* targets, const float* m,
                                const float* l, const float* zt, int64_t N, int64_t V_total,
                                float* stat, float* telemetry, float* objective, float* count,
                                void* stream);

/* Workspace bytes of algx_head_bwd: one bf16 dz slab of N x min(6656, V
 * rounded up to 256), when dh is bf16 an fp32 dh accumulator, and 256 bytes
 * for the slab GEMMs' two tile counters (reset by the kernels themselves; the
 * workspace needs no initialisation). The reference writes dz for the whole
 * vocabulary (fused_head.py:194-216). */
ALGX_API size_t algx_head_bwd_workspace_size(int64_t N, int64_t d, int64_t V, int32_t dh_dtype);

/* dh (N, d) in dh_dtype (partial over this rank's vocabulary rows) and
 * dembed (V, d) fp32, with scale = g * slope / count read from device
 * memory. The logits are recomputed one vocabulary slab of at most 6656
 * columns at a time (never in full): a tcgen05 kernel writes the slab's
 * bf16 dz = scale * (softmax - y) or scale * (p - y) r into the workspace,
 * then one persistent tcgen05 GEMM launch computes dE_slab = dz^T . h and
 * dh += dz . E_slab (fp32 accumulation). Replaces kernels/fused_head.py:120-156, 194-216
 * (`_bwd_kernel`, `_backward`, including the XLA dE = dz^T h product). */
ALGX_API int algx_head_bwd(const algx_head_config* cfg, const void* h, const void* embed,
                           const int32_t* targets, const float* stat, const float* scale, void* dh,
                           int32_t dh_dtype, float* dembed, int64_t N, int64_t d, int64_t V,
                           int64_t vocab_offset, int32_t dtype, void* workspace, size_t workspace_bytes,
                           void* stream);

/* --------------------------------------------- packed (token-major) attention */
/* The model's QKV projection writes one token-major tensor qkv (B, T, 3, H, D)
 * ([q | k | v] per token, each H x D); its output projection reads the
 * attention output token-major (B, T, H, D). These entries read and write
 * those layouts directly, so no head-major copy of q, k, v or of their
 * gradients is made outside the kernels. No counterpart in the reference:
 * XLA fuses its transposes (model.py:166-169, 180) into neighbouring ops. */

/* algx_qknorm_attn_prepare on the packed qkv: q_scaled and k_norm as there,
 * v_heads = v in head-major order (B, H, T, D) for algx_attn_fwd. */
ALGX_API int algx_qknorm_attn_prepare_packed(const algx_attn_config* cfg, const void* qkv, const float* gain_q,
                                             const float* gain_k, const float* rope_cos, const float* rope_sin,
                                             int64_t rope_rows, const float* sink, void* q_scaled, void* k_norm,
                                             void* v_heads, float* guard, int64_t B, int64_t H, int64_t T, int64_t D,
                                             int32_t dtype, float eps, void* stream);

/* Workspace bytes of algx_qknorm_attn_bwd_packed: that of
 * algx_qknorm_attn_bwd plus head-major dq, dk, dv scratch. No counterpart in the reference: XLA sizes the Pallas kernels' scratch itself. */
ALGX_API size_t algx_qknorm_attn_bwd_packed_workspace_size(int64_t B, int64_t H, int64_t T, int64_t D,
                                                           int32_t dtype);

/* algx_qknorm_attn_bwd for a forward run by algx_qknorm_attn_prepare_packed:
 * dout head-major (B, H, T, D); dqkv (B, T, 3, H, D) receives the gradients of
 * the raw q and k and of v in the packed layout. Replaces the backward of
 * model.py:166-180 (projections' transposes, QK norm, rotary, flash.py:718-726). */
ALGX_API int algx_qknorm_attn_bwd_packed(const algx_attn_config* cfg, const void* qkv, const float* gain_q,
                                         const float* gain_k, const float* rope_cos, const float* rope_sin,
                                         int64_t rope_rows, const void* q_scaled, const void* k_norm,
                                         const void* v_heads, const float* sink, const float* guard, const void* o,
                                         const float* o_precise, const float* stat, const void* dout, void* dqkv,
                                         float* dgain_q, float* dgain_k, float* dsink, int64_t B, int64_t H,
                                         int64_t T, int64_t D, int32_t dtype, float eps, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* dst (B, T, H, D) = src (B, H, T, D) and back, D = 64, src != dst: the
 * attention output into the output projection and its gradient out of it
 * (model.py:180). No counterpart in the reference (an XLA transpose). */
ALGX_API int algx_heads_to_tokens(const void* src, void* dst, int64_t B, int64_t H, int64_t T, int64_t D,
                                  int32_t dtype, void* stream);
/* The inverse permutation: dO from the output projection back to head-major
 * order. No counterpart in the reference (an XLA transpose). */
ALGX_API int algx_tokens_to_heads(const void* src, void* dst, int64_t B, int64_t H, int64_t T, int64_t D,
                                  int32_t dtype, void* stream);

/* ------------------------------------------------ training-step elementwise */
/* The model's own row norms and gate around the hot kernels, used by the
 * config-5 training step (algx.model). bf16 or fp32 rows, fp32 maths. */

/* y = rms_norm(x) * gain over rows of `dim` elements (dim a multiple of 16
 * bytes, at most 4096 bf16 / 2048 fp32); gain NULL gives the parameter-free
 * form. Replaces algebraic.py:76-83 `rms_norm` as the model calls it
 * (model.py:158-159 `_norm`: ln1, ln2, embed_gain, final_gain). */
ALGX_API int algx_rmsnorm_fwd(const void* x, const float* gain, void* y, int64_t rows, int64_t dim,
                              int32_t dtype, float eps, void* stream);

/* Bytes of workspace algx_rmsnorm_bwd needs (one fp32 row of dgain partials
 * per CTA). No counterpart in the reference (XLA reduces dgain itself). */
ALGX_API size_t algx_rmsnorm_bwd_workspace_size(int64_t rows, int64_t dim);

/* dx and dgain of algx_rmsnorm_fwd (JAX AD of algebraic.py:76-83 in the
 * reference's training step, model.py:158-159). dgain is summed in a fixed
 * order (deterministic). gain NULL: no dgain, no workspace needed. */
ALGX_API int algx_rmsnorm_bwd(const void* x, const float* gain, const void* dy, void* dx, float* dgain,
                              int64_t rows, int64_t dim, int32_t dtype, float eps, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Residual add fused into the following norm (model.py:180-200): s = x + r
 * rounded to the I/O dtype, written to s_out, and y = rms_norm(s) * gain as
 * algx_rmsnorm_fwd. No counterpart in the reference (XLA fuses the add). */
ALGX_API int algx_add_rmsnorm_fwd(const void* x, const void* r, const float* gain, void* s_out, void* y,
                                  int64_t rows, int64_t dim, int32_t dtype, float eps, void* stream);

/* Backward of algx_add_rmsnorm_fwd: dx = (norm backward of dy at s) + ds,
 * rounded once, where ds is the gradient reaching s from its other consumer;
 * dx is the gradient of both x and r. Workspace as algx_rmsnorm_bwd. No
 * counterpart in the reference (JAX AD of the add and norm, model.py:180-200). */
ALGX_API int algx_add_rmsnorm_bwd(const void* s, const float* gain, const void* dy, const void* ds, void* dx,
                                  float* dgain, int64_t rows, int64_t dim, int32_t dtype, float eps, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* y = gate * silu(up), bf16, for rows of gu = [gate (ff) | up (ff)]; y is
 * (rows, ff). ff a multiple of 8. Replaces model.py:193-198 (`gate * act`,
 * act = S.silu(up), standard.py:12-13), evaluated in fp32 and rounded once. */
ALGX_API int algx_swiglu_fwd(const void* gu, void* y, int64_t rows, int64_t ff, void* stream);

/* dgu = [dgate | dup] of algx_swiglu_fwd for the upstream gradient dy
 * (rows, ff); JAX AD of model.py:193-198. */
ALGX_API int algx_swiglu_bwd(const void* gu, const void* dy, void* dgu, int64_t rows, int64_t ff, void* stream);

/* y = gate * alu(up, beta), bf16, for rows of gu = [gate (ff) | up (ff)]:
 * the algebraic preset's feed-forward gate (model.py:196-197). alu is
 * algebraic.py:86-101 (rounded to bf16 as `_alu_parts` does), the product
 * is rounded once more. */
ALGX_API int algx_aluglu_fwd(const void* gu, void* y, int64_t rows, int64_t ff, float beta, void* stream);

/* dgu = [dgate | dup] of algx_aluglu_fwd with the reference's custom VJP of
 * alu (algebraic.py:104-113). */
ALGX_API int algx_aluglu_bwd(const void* gu, const void* dy, void* dgu, int64_t rows, int64_t ff, float beta,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ALGX_H_ */
