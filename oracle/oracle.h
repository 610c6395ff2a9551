/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's host arithmetic for the non-GEMM
 * extension-op path of tenferro-decision-rs (AtelierArith/tenferro-decision-rs):
 *   - crates/cpu-kernels/src/lib.rs       (f32 kernels; the in-repo, pinned arithmetic)
 *   - crates/tenferro-ext/src/lib.rs      (f64 erf, gelu_erf composition)
 *   - crates/tenferro-infer/src/{norm,softmax,rope}.rs (f64 / composite semantics)
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs load
 * this library, and only as the checker / the timed CPU baseline. The product
 * (libtfx.so) never links, loads or calls it.
 *
 * Parity pins: the restatement is checked against every known-answer test the
 * reference holds for this path (crates/tenferro-ext/tests/erf.rs,
 * crates/tenferro-ext/src/layernorm.rs tests, crates/cpu-kernels/src/lib.rs
 * tests, crates/tenferro-infer/tests/primitives.rs); see tests/golden/.
 * Bit-level agreement with the compiled Rust cannot be observed here (no Rust
 * toolchain), so the f32 kernels are restated operation by operation:
 * Rust `mul_add` -> fmaf, sequential f32 sums in the same order, glibc
 * expf/exp2f/sqrtf, no floating-point contraction (-ffp-contract=off).
 */
#ifndef TFX_ORACLE_H
#define TFX_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- thread pool (restates rayon's data-parallel splits) ------------- */
void orc_set_threads(int threads);
int orc_threads(void);

/* ---- crates/cpu-kernels/src/lib.rs (f32) ------------------------------ */
float orc_erf_f32(float a);          /* lib.rs:449-471 */
float orc_expm1_mlx_f32(float a);    /* lib.rs:474-505 */
float orc_gelu_erf_f32(float x);     /* lib.rs:509-511 */
void orc_erf_f32_n(const float* x, float* y, int64_t n);
void orc_gelu_erf_f32_n(const float* x, float* y, int64_t n);

void orc_layer_norm_feature_first_f32(const float* x, int64_t d, int64_t cols,
                                      const float* weight, const float* bias /* nullable */,
                                      float eps, float* y);            /* lib.rs:397-443 */
void orc_geglu_f32(const float* u, int64_t inter, int64_t cols, float* out); /* lib.rs:516-538 */
void orc_rms_norm_last_f32(const float* x, int64_t rows, int64_t width,
                           const float* weight, int centered, float eps, float* out); /* lib.rs:545-581 */
void orc_gated_silu_f32(const float* gate, const float* up, float* out, int64_t n); /* lib.rs:584-607 */
/* Epilogue of input_mul_weight_transpose_bias_into (lib.rs:274-288): y[o + F*t] = x[o + F*t] + bias[o]. */
void orc_bias_add_f32(const float* x, const float* bias, float* y, int64_t features, int64_t tokens);
/* FusedScope::bias_act_first semantics (cuda_fused.rs:704-745) with the cpu-kernels GELU:
 * act 0 = identity, 1 = gelu_erf_f32, 2 = relu. */
void orc_bias_act_f32(const float* x, const float* bias /* nullable */, float* y,
                      int64_t features, int64_t tokens, int act);
/* Full gemm_bias op, restated naively: y (out, length) = bias as the initial
 * accumulator, then += sum_i x[i + in*t] * w[i + in*o] ... see oracle.cpp. */
void orc_gemm_bias_f32(const float* x, const float* weight, const float* bias, float* y,
                       int64_t in_dim, int64_t out_dim, int64_t length);
/* residual add of the layer chain: y = a + b */
void orc_add_f32(const float* a, const float* b, float* y, int64_t n);

/* Masked row softmax over rows of a row-major [batch][heads][q_len][k_len]
 * score tensor (keys contiguous).
 *   semantics 0 (EXCLUDE): cpu-kernels attention rows (lib.rs:1053-1080,
 *     1111-1153): masked -> -inf, p = isfinite(v) ? exp(v - max) : 0,
 *     sequential sum, p / sum (an empty row gives NaN).
 *   semantics 1 (FILL): tenferro-infer masked_softmax (softmax.rs:26-34,
 *     util.rs:87): masked -> -1e30, plain softmax (an empty row is uniform).
 * v = s * scale (+ add_mask); keep = causal / window / valid_len / keep mask. */
void orc_masked_softmax_f32(const float* scores, float* probs,
                            int64_t batch, int64_t heads, int64_t q_len, int64_t k_len,
                            float scale, int semantics, int causal, int64_t window,
                            int window_skips_invalid_query, int64_t valid_len,
                            const int32_t* valid_lens /* nullable, [batch] */,
                            const float* add_mask, int64_t add_sb, int64_t add_sq, int64_t add_sk,
                            const uint8_t* keep, int64_t keep_sb, int64_t keep_sq, int64_t keep_sk);

/* RoPE tables per tenferro-infer rope.rs:84-92: angle computed in f64,
 * cos/sin rounded to f32. Row-major (seq, rotary_dim/2): cos[p*half + i]. */
void orc_rope_tables_f32(double base, int64_t seq, int64_t rotary_dim, float* cos_t, float* sin_t);
void orc_rope_tables_f64(double base, int64_t seq, int64_t rotary_dim, double* cos_t, double* sin_t);
/* rotate_pair_half (rope.rs:68-113) over a strided x: element (v, p, b, j) at
 * v*s_vec + p*s_pos + b*s_batch + j*s_feat; channels j >= rotary_dim copied. */
void orc_rope_pairhalf_f32(const float* x, float* y, const float* cos_t, const float* sin_t,
                           int64_t n_vec, int64_t seq, int64_t batch, int64_t head_dim,
                           int64_t rotary_dim, int64_t s_vec, int64_t s_pos, int64_t s_batch,
                           int64_t s_feat);
void orc_rope_pairhalf_f64(const double* x, double* y, const double* cos_t, const double* sin_t,
                           int64_t n_vec, int64_t seq, int64_t batch, int64_t head_dim,
                           int64_t rotary_dim, int64_t s_vec, int64_t s_pos, int64_t s_batch,
                           int64_t s_feat);

/* ---- attention blocks (crates/cpu-kernels/src/lib.rs) ------------------ */
/* RoPE tables as cpu-kernels builds them, in f32: angle = (p as f32) *
 * base.powf(-2 i / rotary_dim) with glibc powf, then cosf / sinf
 * (lib.rs:938-946 Laya, :696-699 Jeff). Row-major (seq, rotary_dim/2). */
void orc_rope_tables_powf_f32(float base, int64_t seq, int64_t rotary_dim, float* cos_t,
                              float* sin_t);
/* Laya split + RoPE (lib.rs:972-1009): qkv feature-first (3d, L, B) -> head-major
 * (B, heads, L, hd) q/k/v; cos_t/sin_t (L, hd/2) or null for no RoPE. */
void orc_laya_qkv_prep_f32(const float* qkv, const float* cos_t, const float* sin_t,
                           int64_t hidden, int64_t heads, int64_t length, int64_t batch,
                           float* qh, float* kh, float* vh);
/* The fused Laya attention block (laya_attention_block_into, lib.rs:819-1150,
 * scalar path): split, RoPE, masked scaled dot-product attention, out (d, L, B).
 * keep (L, L, B) with element query + L*(key + L*b); an all-masked row is NaN. */
void orc_laya_attention_block_f32(const float* qkv, const uint8_t* keep, int64_t hidden,
                                  int64_t heads, int64_t length, int64_t batch,
                                  const float* cos_t, const float* sin_t, float* out);
/* Jeff prep (lib.rs:660-709): per head centred RMSNorm of q and k over head_dim
 * (mean of squares divided by head_dim, x * (scale * (1 + w))), partial RoPE on
 * the first rotary_dim channels; v copied. q, k, v (length, heads*head_dim)
 * column-major; outputs head-major (heads, length, head_dim). */
void orc_jeff_qkv_prep_f32(const float* q, const float* k, const float* v, const float* q_norm,
                           const float* k_norm, const float* cos_t, const float* sin_t,
                           int64_t length, int64_t heads, int64_t head_dim, int64_t rotary_dim,
                           float eps, float* qh, float* kh, float* vh);
/* jeff_full_attention_into (lib.rs:618-760): prep, causal attention over keys
 * with mask[key] != 0, sigmoid gate; out (length, width); an all-masked row is 0.
 * Tables are built inside with powf (theta, rotary_dim). */
void orc_jeff_full_attention_f32(const float* q, const float* k, const float* v,
                                 const float* gate, const float* q_norm, const float* k_norm,
                                 const float* mask, int64_t length, int64_t heads,
                                 int64_t head_dim, int64_t rotary_dim, float theta, float eps,
                                 float* out);

/* Token embedding gather (fused.cu:304-318): out(t, f) = table(f, ids[t]) with
 * table element (f, id) at f*t_feat + id*t_tok and out element (t, f) at
 * t*o_tok + f*o_feat (ids already validated). */
void orc_embedding_f32(const float* table, const int64_t* ids, float* out, int64_t hidden,
                       int64_t length, int64_t o_tok, int64_t o_feat, int64_t t_feat,
                       int64_t t_tok);

/* ---- f64 composites (tenferro-infer, tenferro-ext lib.rs) ---------- */
double orc_erf_f64(double x);                                   /* tenferro-ext lib.rs:273-285 */
void orc_erf_f64_n(const double* x, double* y, int64_t n);
void orc_gelu_erf_f64_n(const double* x, double* y, int64_t n); /* tenferro-ext lib.rs:224-234 */
void orc_layer_norm_feature_first_f64(const double* x, int64_t d, int64_t cols,
                                      const double* weight, const double* bias,
                                      double eps, double* y);   /* norm.rs:11-45 */
void orc_rms_norm_last_f64(const double* x, int64_t rows, int64_t width,
                           const double* weight, int centered, double eps, double* out); /* norm.rs:52-103 */
void orc_softmax_rows_f64(const double* x, double* y, int64_t rows, int64_t cols); /* softmax.rs:8-21 */

#ifdef __cplusplus
}
#endif

#endif /* TFX_ORACLE_H */
