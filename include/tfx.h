/*
 * tfx.h -- C ABI of the B200 (sm_100a) non-GEMM extension ops of
 * tenferro-decision (feature-first LayerNorm, feature-last RMSNorm, exact-erf
 * GELU / GeGLU, gated SiLU, the gemm_bias bias-broadcast epilogue, masked row
 * softmax, RoPE).
 *
 * Library: tenferro-decision-rs_b200/lib/libtfx.so (built with nvcc for
 * sm_100a; links the CUDA runtime statically).
 *
 * Conventions, kept from the reference's extension ops
 * (crates/tenferro-ext/src, crates/tenferro-infer/src):
 *   - Layouts are the reference's column-major ones (first axis fastest).
 *     A feature-first activation (d, cols) stores column c at [c*d, (c+1)*d).
 *   - Inputs are borrowed, outputs are caller-owned. Calls that need scratch
 *     (named at each) allocate it stream-ordered on the call's stream, from a
 *     per-device memory pool that libtfx owns (it keeps up to 1 GiB of freed
 *     scratch mapped between calls; the caller's default pool is not
 *     touched), and release it there; every other call allocates nothing.
 *   - Every call is asynchronous on the given stream (NULL = legacy default
 *     stream) and takes device pointers, except the tfx_session_* calls,
 *     which take host pointers and return when the host outputs are written.
 *   - Errors are returned, never hidden: there is no CPU fallback and no
 *     implicit transfer (crates/tenferro-ext/src/lib.rs:188-189). On failure
 *     tfx_last_error_string() names the op and field the way the reference's
 *     invalid_argument(op, field, message) does, e.g.
 *     "tenferro-ext::layernorm_ff: weight: null pointer".
 *   - An empty tensor (a zero extent) is a successful no-op, as in the
 *     cpu-kernels functions (e.g. crates/cpu-kernels/src/lib.rs:410-412).
 *   - Elementwise ops accept y == x (in place); other overlaps are rejected
 *     where the op would read what it already wrote.
 *   - All functions are thread-safe; the only shared state is a per-device
 *     attribute cache initialised once per device.
 */
#ifndef TFX_H
#define TFX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TFX_API __attribute__((visibility("default")))
#else
#define TFX_API
#endif

/* Same object as cudaStream_t / CUstream (driver_types.h). */
typedef struct CUstream_st* tfx_stream_t;

#define TFX_OK 0
#define TFX_ERR_INVALID_ARGUMENT (-1) /* bad pointer, size or parameter */
#define TFX_ERR_UNSUPPORTED (-2)      /* shape/dtype/layout this build does not handle */
#define TFX_ERR_CUDA (-3)             /* a CUDA runtime call or launch failed */

/* Thread-local description of the last failure on this thread ("" if none). */
TFX_API const char* tfx_last_error_string(void);
/* ABI version: major * 10000 + minor * 100 + patch. */
TFX_API int tfx_version(void);
/* Diagnostic, no counterpart in the reference: the number of bounded waits
 * inside libtfx kernels on the current device that gave up since the library
 * was loaded (a kernel that gives up leaves its output incomplete). Every wait
 * of a kernel on an asynchronous copy or tensor-core operation (the TMA-
 * pipelined RMSNorm, the tensor-core attention and GEMM epilogue) is bounded
 * (about one second),
 * so a lost copy ends the kernel instead of hanging the GPU. Synchronous
 * (reads device memory). */
TFX_API int tfx_wait_timeouts(uint32_t* count);

/* ---- erf / exact GELU ------------------------------------------------------
 * Replaces ErfOp (crates/tenferro-ext/src/lib.rs:95-170) and
 * EagerSessionErfExt::{erf, gelu_erf} (lib.rs:201-234).
 * f32: the MLX erf of crates/cpu-kernels/src/lib.rs:449-505, bit-identical;
 *      GELU = (0.5 * x) * (1 + erf(x * FRAC_1_SQRT_2)) (lib.rs:509-511).
 * f64: Abramowitz-Stegun 7.1.26 (lib.rs:273-285); GELU composed as
 *      (x * 0.5) * (erf(x * FRAC_1_SQRT_2) + 1) (lib.rs:224-234). */
TFX_API int tfx_erf_f32(const float* x, float* y, int64_t n, tfx_stream_t stream);
TFX_API int tfx_gelu_erf_f32(const float* x, float* y, int64_t n, tfx_stream_t stream);
TFX_API int tfx_erf_f64(const double* x, double* y, int64_t n, tfx_stream_t stream);
TFX_API int tfx_gelu_erf_f64(const double* x, double* y, int64_t n, tfx_stream_t stream);

/* ---- GeGLU ---------------------------------------------------------------
 * Replaces GegluOp (crates/tenferro-ext/src/geglu.rs:27,85-121) and
 * FusedScope::geglu_first (crates/tenferro-ext/src/cuda_fused.rs:669).
 * u is feature-first (2*inter, cols); y is (inter, cols):
 *   y[i + inter*c] = gelu_erf(u[i + 2*inter*c]) * u[inter + i + 2*inter*c]
 * (cpu-kernels lib.rs:516-538). y must not overlap u. */
TFX_API int tfx_geglu_ff_f32(const float* u, float* y, int64_t inter, int64_t cols,
                     tfx_stream_t stream);

/* ---- gated SiLU ----------------------------------------------------------
 * Replaces GatedSiluOp (crates/tenferro-ext/src/gated_silu.rs:26,67-106),
 * FusedScope::gated_silu (cuda_fused.rs:640): y = (g / (1 + exp(-g))) * u
 * (cpu-kernels lib.rs:584-607). y may equal gate or up. */
TFX_API int tfx_gated_silu_f32(const float* gate, const float* up, float* y, int64_t n,
                       tfx_stream_t stream);
/* FusedScope::gated_silu_stacked (cuda_fused.rs:995): gu is column-major
 * (rows, 2*inter) with column blocks gate | up; y is (rows, inter). */
TFX_API int tfx_gated_silu_stacked_f32(const float* gu, float* y, int64_t rows, int64_t inter,
                               tfx_stream_t stream);

/* ---- bias broadcast (gemm_bias epilogue) ---------------------------------
 * The bias step of GemmBiasOp (crates/tenferro-ext/src/gemm_bias.rs:27,76-142;
 * cpu-kernels lib.rs:274-288) on a finished product, and
 * FusedScope::bias_act_first (cuda_fused.rs:704): x, y are feature-first
 * (features, tokens) -- equivalently row-major [tokens][features] --
 *   y[o + features*t] = act(x[o + features*t] + bias[o])
 * act: TFX_ACT_IDENTITY, TFX_ACT_GELU_ERF (the f32 GELU above), TFX_ACT_RELU.
 * bias may be NULL (activation only). y may equal x. */
#define TFX_ACT_IDENTITY 0
#define TFX_ACT_GELU_ERF 1
#define TFX_ACT_RELU 2
TFX_API int tfx_bias_act_ff_f32(const float* x, const float* bias, float* y, int64_t features,
                        int64_t tokens, int act, tfx_stream_t stream);

/* ---- GEMM with a fused epilogue ---------------------------------------------
 * The MLP projection with its epilogue in the same kernel (tcgen05 tensor
 * cores, 3xTF32 for f32 accuracy; the projection never reaches HBM).
 * x is feature-first (in_dim, length), weight is column-major (in_dim, out)
 * -- element (i, o) at i + in_dim*o, the reference's layout --, bias is
 * (out) or NULL:
 *   p[o, t] = bias[o] + sum_i x[i + in_dim*t] * weight[i + in_dim*o]
 * (cpu-kernels lib.rs:274-288 input_mul_weight_transpose_bias_into; 0
 * instead of bias[o] when bias is NULL, input_mul_weight_transpose_into,
 * lib.rs:257-267).
 * tfx_gemm_geglu_ff_f32 replaces GemmGegluOp / EagerSessionGemmGegluExt::
 * gemm_geglu (crates/tenferro-ext/src/gemm_geglu.rs:25-31,114-240,
 * 268-310): out = 2*intermediate, y is (intermediate, length) with
 *   y[j + intermediate*t] = gelu_erf(p[j, t]) * p[intermediate + j, t]
 * (geglu_into, lib.rs:516-538, the f32 GELU above).
 * tfx_gemm_bias_act_ff_f32 replaces GemmBiasOp (gemm_bias.rs:27,76-142), and
 * with an activation the reference's GEMM followed by
 * FusedScope::bias_act_first (cuda_fused.rs:704, kernel fused_bias_act,
 * fused.cu:137): y is (out_dim, length), y[o + out_dim*t] = act(p[o, t]),
 * act as tfx_bias_act_ff_f32.
 * Results are within the f32 tolerance of the reference's f32 GEMM (summation
 * order differs); the epilogue arithmetic is the reference's. Tiles of 128
 * tokens holding a non-finite value (or |v| >= 2^60), and every tile when
 * the weight does, are computed with the reference's sequential arithmetic so
 * that inf / NaN propagate as there. y must not overlap x, weight or bias.
 * Scratch (hi / lo copies of x and weight, about 8 * (in_dim rounded up to
 * 32) * (length + out) bytes) is allocated stream-ordered and released on the
 * stream. */
TFX_API int tfx_gemm_geglu_ff_f32(const float* x, const float* weight, const float* bias,
                                  float* y, int64_t in_dim, int64_t intermediate,
                                  int64_t length, tfx_stream_t stream);
TFX_API int tfx_gemm_bias_act_ff_f32(const float* x, const float* weight, const float* bias,
                                     float* y, int64_t in_dim, int64_t out_dim, int64_t length,
                                     int act, tfx_stream_t stream);

/* Residual add of the encoder layer (laya-infer/src/model.rs add_assign):
 * y = a + b elementwise. y may equal a or b. */
TFX_API int tfx_add_f32(const float* a, const float* b, float* y, int64_t n, tfx_stream_t stream);

/* ---- feature-first LayerNorm ---------------------------------------------
 * Replaces LayerNormFeatureFirstOp (crates/tenferro-ext/src/layernorm.rs:33,
 * 94-231), EagerSessionLayerNormExt::layer_norm_feature_first (:260) and
 * FusedScope::layer_norm_first (cuda_fused.rs:603).
 * x, y are (d, cols), column c contiguous; weight and bias (nullable) are (d).
 *   mean = sum(x)/d; var = sum((x-mean)^2)/d; inv = 1/sqrt(var + eps);
 *   y = (x - mean) * inv * w (+ b)              (cpu-kernels lib.rs:397-443)
 * f64 restates tenferro_infer::norm::layer_norm (norm.rs:11-45) on the same
 * layout. y may equal x. */
TFX_API int tfx_layernorm_ff_f32(const float* x, const float* weight, const float* bias, float* y,
                         int64_t d, int64_t cols, float eps, tfx_stream_t stream);
TFX_API int tfx_layernorm_ff_f64(const double* x, const double* weight, const double* bias, double* y,
                         int64_t d, int64_t cols, double eps, tfx_stream_t stream);

/* ---- feature-last RMSNorm -------------------------------------------------
 * Replaces RmsNormLastOp (crates/tenferro-ext/src/rms_norm.rs:28,84-137),
 * EagerSessionRmsNormExt::rms_norm_last (:165-203) and
 * FusedScope::rms_norm_last (cuda_fused.rs:575).
 * x, y are column-major (rows, width): element (r, d) at r + rows*d.
 *   scale = 1/sqrt(sum_d x^2 * (1/width) + eps); y = x * scale * (centered ? 1+w : w)
 * (cpu-kernels lib.rs:545-581; the eps of the ext trait is an f64 truncated
 * to f32, rms_norm.rs:186 -- pass the truncated value). f64 restates
 * tenferro_infer::norm::rms_norm (norm.rs:52-103). y may equal x. */
TFX_API int tfx_rmsnorm_last_f32(const float* x, const float* weight, float* y, int64_t rows,
                         int64_t width, int centered, float eps, tfx_stream_t stream);
TFX_API int tfx_rmsnorm_last_f64(const double* x, const double* weight, double* y, int64_t rows,
                         int64_t width, int centered, double eps, tfx_stream_t stream);
/* Same result as tfx_rmsnorm_last_f32, for callers that cannot let a library
 * allocate device memory during a call -- e.g. a serving process whose HBM is
 * reserved up front by its own allocator, or a latency-critical loop that must
 * not touch an allocator or risk an allocation's implicit synchronisation.
 * No counterpart in the reference. It allocates and frees nothing: the
 * kernels' partial sums live in a fixed 4 MiB array inside libtfx's device
 * image, reserved on every GPU that loads the library until the process
 * exits. Limit: rows * ceil(width / 64) <= 1048576 (e.g. width 1024: up to
 * 65536 rows; width 4096: up to 16384); larger calls return
 * TFX_ERR_UNSUPPORTED. The first call on a device looks the array up for that
 * device (make it before any stream capture). All calls share the array, so
 * calls that can overlap on the GPU (other streams, other threads) race and
 * must be serialised by the caller; nothing in it needs clearing between
 * calls. */
TFX_API int tfx_rmsnorm_last_f32_noalloc(const float* x, const float* weight, float* y,
                                         int64_t rows, int64_t width, int centered, float eps,
                                         tfx_stream_t stream);

/* ---- masked row softmax ---------------------------------------------------
 * Replaces tenferro_infer::softmax::{softmax, masked_softmax}
 * (crates/tenferro-infer/src/softmax.rs:8-34) and the masked softmax rows
 * inside the attention kernels (cpu-kernels lib.rs:1053-1080, 1111-1153;
 * fused.cu fused_attention). Scores are row-major
 * [batch][heads][q_len][k_len], keys contiguous; probabilities have the same
 * layout (y may equal scores).
 * For query q of batch b, key k is kept when all enabled conditions hold:
 *   valid:  k < valid_len (or valid_lens[b] when valid_lens != NULL)
 *   causal: k <= q
 *   window: |q - k| <= window  (skipped for q >= the valid length when
 *           window_skips_invalid_query, as laya-infer/src/model.rs:474-483)
 *   keep:   keep[b*keep_stride_b + q*keep_stride_q + k*keep_stride_k] != 0
 * and the score is v = s * scale (+ add_mask[b*sb + q*sq + k*sk]).
 * semantics TFX_SOFTMAX_EXCLUDE: masked keys are -inf, non-finite values
 *   contribute 0, p = exp(v - max) / sum; an all-masked row is NaN
 *   (cpu-kernels attention rows).
 * semantics TFX_SOFTMAX_FILL: masked keys are filled with -1e30 and a plain
 *   softmax follows; an all-masked row is uniform (tenferro-infer
 *   masked_softmax, util.rs:87). */
#define TFX_SOFTMAX_EXCLUDE 0
#define TFX_SOFTMAX_FILL 1
typedef struct tfx_softmax_desc {
  int64_t batch, heads, q_len, k_len;
  float scale;                   /* 1.0f = scores used as given */
  int32_t semantics;             /* TFX_SOFTMAX_EXCLUDE or TFX_SOFTMAX_FILL */
  int32_t causal;                /* nonzero: keep k <= q */
  int32_t window_skips_invalid_query;
  int64_t window;                /* < 0: no window */
  int64_t valid_len;             /* < 0: all keys valid (ignored when valid_lens != NULL) */
  const int32_t* valid_lens;     /* nullable device array [batch] */
  const float* add_mask;         /* nullable device additive mask */
  int64_t add_stride_b, add_stride_q, add_stride_k;
  const uint8_t* keep;           /* nullable device boolean mask */
  int64_t keep_stride_b, keep_stride_q, keep_stride_k;
} tfx_softmax_desc;
/* Fills a descriptor for an unmasked softmax over rows of length k_len. */
TFX_API void tfx_softmax_desc_init(tfx_softmax_desc* desc, int64_t batch, int64_t heads,
                           int64_t q_len, int64_t k_len);
TFX_API int tfx_masked_softmax_f32(const float* scores, float* probs, const tfx_softmax_desc* desc,
                           tfx_stream_t stream);

/* ---- RoPE -----------------------------------------------------------------
 * Replaces tenferro_infer::rope::{rope_modernbert, rope_qwen_partial}
 * (crates/tenferro-infer/src/rope.rs:36-66, rotate_pair_half :68-113) and the
 * RoPE step of FusedScope::laya_attention / jeff_attention.
 * x, y are strided: element (vec v, position p, batch b, channel j) at
 * v*stride_vec + p*stride_pos + b*stride_batch + j*stride_feat. Pairs are
 * (i, i + rotary_dim/2) for i < rotary_dim/2:
 *   y_i = x_i*cos - x_{i+half}*sin,  y_{i+half} = x_i*sin + x_{i+half}*cos
 * each product rounded separately; channels j >= rotary_dim are copied.
 * cos/sin are device tables (seq, rotary_dim/2), row-major, for positions
 * 0..seq-1, e.g. from tfx_rope_tables_f32. y may equal x. */
typedef struct tfx_rope_desc {
  int64_t n_vec, seq, batch, head_dim, rotary_dim;
  int64_t stride_vec, stride_pos, stride_batch, stride_feat;
} tfx_rope_desc;
TFX_API int tfx_rope_pairhalf_f32(const float* x, float* y, const float* cos_table,
                          const float* sin_table, const tfx_rope_desc* desc,
                          tfx_stream_t stream);
/* Host helper (no GPU): the reference's tables, angle p * base^(-2i/rotary_dim)
 * in f64, cos/sin rounded to f32 (rope.rs:84-92, table() :15-24). Host arrays
 * of seq * rotary_dim/2 floats. */
TFX_API int tfx_rope_tables_f32(double base, int64_t seq, int64_t rotary_dim, float* cos_host,
                        float* sin_host);

/* ---- residual add fused into LayerNorm ------------------------------------------
 * The chain's residual add followed by a feature-first LayerNorm as one pass
 * (the "residual-add + LayerNorm" epilogue fusion; the reference runs the two
 * ops separately, laya-infer's residual add then LayerNormFeatureFirstOp,
 * crates/tenferro-ext/src/layernorm.rs:33-231). s = a + b (each sum rounded),
 * y = LayerNorm(s) with tfx_layernorm_ff_f32's arithmetic: bit-identical to
 * tfx_add_f32 then tfx_layernorm_ff_f32. s is written to sum_out when it is
 * non-NULL (the residual stream the next layer needs). sum_out and y may each
 * equal a or b exactly but not overlap them partially or each other. */
TFX_API int tfx_add_layernorm_ff_f32(const float* a, const float* b, const float* weight,
                                     const float* bias, float* sum_out, float* y, int64_t d,
                                     int64_t cols, float eps, tfx_stream_t stream);

/* ---- token embedding gather ------------------------------------------------------
 * FusedScope::embedding_rows / embedding_columns (crates/tenferro-ext/src/
 * cuda_fused.rs:817-898; kernel fused.cu:304-318): out(token t, feature f) =
 * table(feature f, ids[t]).
 *   TFX_EMBED_ROWS:    table row-major (hidden, vocab), element (f, id) at
 *                      f*vocab + id; out time-first (length, hidden), (t, f) at
 *                      t + length*f.
 *   TFX_EMBED_COLUMNS: table column-major (hidden, vocab), element (f, id) at
 *                      f + hidden*id; out feature-first (hidden, length), (f, t)
 *                      at f + hidden*t.
 * tfx_embedding_f32 takes the ids on the host, as the reference does, rejects
 * any id outside [0, vocab) before launching (TFX_ERR_INVALID_ARGUMENT naming
 * the first), and copies them into a stream-ordered scratch buffer.
 * tfx_embedding_gather_f32 takes device ids and cannot validate them before
 * launching: an out-of-range id yields a NaN vector (no memory is read out of
 * bounds). */
#define TFX_EMBED_ROWS 0
#define TFX_EMBED_COLUMNS 1
TFX_API int tfx_embedding_f32(const float* table, const int64_t* ids_host, float* out,
                              int64_t hidden, int64_t vocab, int64_t length, int32_t layout,
                              tfx_stream_t stream);
TFX_API int tfx_embedding_gather_f32(const float* table, const int64_t* ids_device, float* out,
                                     int64_t hidden, int64_t vocab, int64_t length,
                                     int32_t layout, tfx_stream_t stream);

/* ---- attention blocks -------------------------------------------------------
 * The attention cores of the two forwards, mirroring the reference's CUDA
 * path (FusedScope::laya_attention / jeff_attention, crates/tenferro-ext/src/
 * cuda_fused.rs:911-993, 1029-1103: a prep kernel writes head-major q, k, v,
 * then one attention kernel, fused.cu:157-306) with the arithmetic of its CPU
 * ops (crates/cpu-kernels/src/lib.rs:618-760 jeff_full_attention_into,
 * :819-1150 laya_attention_block_into, behind LayaAttentionBlockOp,
 * crates/tenferro-ext/src/laya_attention.rs:27-176). Head-major tensors are
 * (batch, heads, length, head_dim) with head_dim contiguous. */

/* Host helper (no GPU): RoPE tables as cpu-kernels builds them, in f32:
 * angle = (p as f32) * base.powf(-2 i / rotary_dim) with the C library's
 * powf, cos/sin by cosf/sinf (lib.rs:938-946, :696-699). Row-major
 * (seq, rotary_dim/2). */
TFX_API int tfx_rope_tables_powf_f32(float base, int64_t seq, int64_t rotary_dim, float* cos_host,
                                     float* sin_host);

/* Laya split + RoPE (lib.rs:972-1009; CUDA twin fused_laya_qkv_prep,
 * fused.cu:199-229): qkv feature-first (3*hidden, length, batch) -> head-major
 * qh, kh, vh; q and k rotated over the full head (pairs i, i + head_dim/2)
 * with device tables (length, head_dim/2), or copied when cos_table is NULL.
 * Results are bit-identical to the reference arithmetic. */
TFX_API int tfx_laya_qkv_prep_f32(const float* qkv, const float* cos_table,
                                  const float* sin_table, float* qh, float* kh, float* vh,
                                  int64_t hidden, int64_t heads, int64_t length, int64_t batch,
                                  tfx_stream_t stream);

/* Jeff prep (lib.rs:660-709; CUDA twin fused_jeff_qkv_prep, fused.cu:150-197):
 * q, k, v (length, heads*head_dim) column-major (time-first) -> head-major
 * (1, heads, length, head_dim). q and k: centred RMSNorm per head over
 * head_dim (mean of squares / head_dim, x * (1/sqrt(m + eps) * (1 + norm))),
 * then RoPE on the first rotary_dim channels (pairs i, i + rotary_dim/2;
 * tables (length, rotary_dim/2), may be NULL when rotary_dim == 0). v copied.
 * Bit-identical to the reference arithmetic (sequential sums per token). */
TFX_API int tfx_jeff_qkv_prep_f32(const float* q, const float* k, const float* v,
                                  const float* q_norm, const float* k_norm,
                                  const float* cos_table, const float* sin_table, float* qh,
                                  float* kh, float* vh, int64_t length, int64_t heads,
                                  int64_t head_dim, int64_t rotary_dim, float eps,
                                  tfx_stream_t stream);

#define TFX_ATTN_EMPTY_NAN 0  /* a row without kept keys is NaN (cpu-kernels Laya) */
#define TFX_ATTN_EMPTY_ZERO 1 /* ... is 0 (fused_attention, cpu-kernels Jeff) */

/* Masked scaled dot-product attention over head-major q, k, v (fused.cu:
 * 231-306 / lib.rs:711-752, 1106-1147). score = (q . k) * scale (+ bias);
 * a key is dropped when causal and key > query, when |query - key| > window
 * (window >= 0), when key >= valid_len (valid_len >= 0), when keep is given
 * and keep[q + L*(k + L*b)] == 0, or when active is given and
 * active[b*L + k] == 0. Scores that are not finite contribute nothing (as
 * the reference's isfinite test); a row without a kept key, or with a +inf
 * score, is NaN or 0 per empty_rows. Output element (token t, feature
 * f = head*head_dim + d, batch b) at t*out_tok + f*out_feat + b*out_batch; with
 * gate it is multiplied by 1/(1 + exp(-gate[gate_offset + that index])). */
typedef struct tfx_attention_desc {
  int64_t batch, heads, length, head_dim;
  float scale;         /* default 1/sqrt(head_dim) */
  int32_t empty_rows;  /* TFX_ATTN_EMPTY_NAN (default) or TFX_ATTN_EMPTY_ZERO */
  int32_t causal;      /* default 0 */
  int64_t window;      /* default -1 (none) */
  int64_t valid_len;   /* default -1 (none) */
  const uint8_t* keep; /* nullable, (length, length, batch), query fastest */
  const float* bias;   /* nullable, same layout, added to the scaled score */
  const float* active; /* nullable, (batch, length) key mask */
  const float* gate;   /* nullable */
  int64_t gate_offset;
  int64_t out_tok, out_feat, out_batch; /* default (heads*head_dim, 1, heads*head_dim*length) */
} tfx_attention_desc;
TFX_API int tfx_attention_desc_init(tfx_attention_desc* desc, int64_t batch, int64_t heads,
                                    int64_t length, int64_t head_dim);
TFX_API int tfx_attention_f32(const float* qh, const float* kh, const float* vh, float* out,
                              const tfx_attention_desc* desc, tfx_stream_t stream);

/* The fused Laya attention block (LayaAttentionBlockOp): prep + attention with
 * cpu-kernels semantics (keep mask, all-masked rows NaN), out (hidden, length,
 * batch). Head-major q, k, v live in a stream-ordered scratch allocation
 * (3 * hidden * length * batch floats) released on the stream. */
TFX_API int tfx_laya_attention_block_f32(const float* qkv, const uint8_t* keep,
                                         const float* cos_table, const float* sin_table,
                                         float* out, int64_t hidden, int64_t heads,
                                         int64_t length, int64_t batch, tfx_stream_t stream);

/* Jeff full attention (jeff_full_attention_into / FusedScope::jeff_attention):
 * prep, causal attention over keys with mask[key] != 0, sigmoid gate (gate
 * (length, width) like q); all-masked rows are 0. out (length, heads*head_dim)
 * column-major. Scratch from the library's stream-ordered pool: with length a
 * multiple of 128, head_dim 64 / 128 / 256, heads*length^2 <= 2^30 and 16-byte
 * aligned gate and out, the tensor-core route (about (6 + s) n + 3 heads
 * length^2 floats, n = length*heads*head_dim, s = the most CTAs (or CTA
 * pairs) one query tile's P V contraction is split over: 3 at 8 heads x 2048
 * tokens);
 * otherwise 3 n floats. */
TFX_API int tfx_jeff_attention_f32(const float* q, const float* k, const float* v,
                                   const float* gate, const float* q_norm, const float* k_norm,
                                   const float* mask, const float* cos_table,
                                   const float* sin_table, float* out, int64_t length,
                                   int64_t heads, int64_t head_dim, int64_t rotary_dim,
                                   float eps, tfx_stream_t stream);

/* ---- host-buffer sessions ---------------------------------------------------
 * The reference executes these ext ops on host tensors of a CPU session
 * (execute_*_in_session over TensorRead slices, e.g.
 * crates/tenferro-ext/src/layernorm.rs:94-231, rms_norm.rs:84-137,
 * geglu.rs:85-121, gated_silu.rs:67-106, gemm_bias.rs:76-142). A session is
 * the drop-in for that executor: same arguments as the device entry points
 * above, but x / y / weights / masks are HOST pointers, and the call returns
 * once the host outputs are written. Work is split into chunks along the
 * token axis and pipelined (copy in, kernel, copy out) over three streams of
 * the session's GPU. Pinned host memory makes the copies fully asynchronous.
 * A session serialises its own calls; use one session per host thread for
 * concurrency, or one per GPU. */
typedef struct tfx_session tfx_session;
TFX_API int tfx_session_create(int device, tfx_session** out);
TFX_API int tfx_session_destroy(tfx_session* session);
/* Target staging bytes (inputs + outputs) per pipelined chunk; default 32 MiB. */
TFX_API int tfx_session_set_chunk_bytes(tfx_session* session, int64_t bytes);
TFX_API int tfx_session_layernorm_ff_f32(tfx_session* session, const float* x,
                                         const float* weight, const float* bias, float* y,
                                         int64_t d, int64_t cols, float eps);
TFX_API int tfx_session_layernorm_ff_f64(tfx_session* session, const double* x,
                                         const double* weight, const double* bias, double* y,
                                         int64_t d, int64_t cols, double eps);
TFX_API int tfx_session_rmsnorm_last_f32(tfx_session* session, const float* x,
                                         const float* weight, float* y, int64_t rows,
                                         int64_t width, int centered, float eps);
TFX_API int tfx_session_erf_f32(tfx_session* session, const float* x, float* y, int64_t n);
TFX_API int tfx_session_gelu_erf_f32(tfx_session* session, const float* x, float* y, int64_t n);
TFX_API int tfx_session_geglu_ff_f32(tfx_session* session, const float* u, float* y,
                                     int64_t inter, int64_t cols);
TFX_API int tfx_session_gated_silu_f32(tfx_session* session, const float* gate,
                                       const float* up, float* y, int64_t n);
TFX_API int tfx_session_bias_act_ff_f32(tfx_session* session, const float* x,
                                        const float* bias, float* y, int64_t features,
                                        int64_t tokens, int act);
TFX_API int tfx_session_add_f32(tfx_session* session, const float* a, const float* b, float* y,
                                int64_t n);
/* tfx_add_layernorm_ff_f32 on host buffers (sum_out may be NULL). */
TFX_API int tfx_session_add_layernorm_ff_f32(tfx_session* session, const float* a,
                                             const float* b, const float* weight,
                                             const float* bias, float* sum_out, float* y,
                                             int64_t d, int64_t cols, float eps);
/* tfx_gemm_geglu_ff_f32 / tfx_gemm_bias_act_ff_f32 on host buffers (the
 * executor of GemmGegluOp / GemmBiasOp on a CPU session's tensors): the weight
 * and bias are uploaded once per call, x and y move in chunks of tokens. */
TFX_API int tfx_session_gemm_geglu_ff_f32(tfx_session* session, const float* x,
                                          const float* weight, const float* bias, float* y,
                                          int64_t in_dim, int64_t intermediate, int64_t length);
TFX_API int tfx_session_gemm_bias_act_ff_f32(tfx_session* session, const float* x,
                                             const float* weight, const float* bias, float* y,
                                             int64_t in_dim, int64_t out_dim, int64_t length,
                                             int act);
/* desc->valid_lens / add_mask / keep are host pointers here. */
TFX_API int tfx_session_masked_softmax_f32(tfx_session* session, const float* scores,
                                           float* probs, const tfx_softmax_desc* desc);
/* Tables are built from base as tfx_rope_tables_f32 does (and cached). The
 * described vectors of y are those of x rotated (channels past rotary_dim
 * copied), as tfx_rope_pairhalf_f32 writes them. Elements of y that belong to
 * no described vector (e.g. the v block of a qkv tensor) are left unchanged
 * when y == x and are otherwise unspecified: when the vectors of a position
 * are contiguous channels at the start of evenly pitched rows (stride_feat 1;
 * q and k of a feature-first qkv tensor, or q alone) only they are copied, as
 * 2-D copies; other layouts copy each batch item's whole extent. */
TFX_API int tfx_session_rope_pairhalf_f32(tfx_session* session, const float* x, float* y,
                                          double base, const tfx_rope_desc* desc);

#ifdef __cplusplus
}
#endif

#endif /* TFX_H */
