// softmax.cu -- masked row softmax over row-major [batch][heads][q_len][k_len]
// scores (keys contiguous).
//
// A group of 8, 16 or 32 lanes owns one row of up to 1024 keys: the row is read
// once with 128-bit loads into registers, the max and the sum are shuffle
// reductions over registers, and the probabilities are written once. Longer rows use a CTA per
// row (up to 8192 keys in registers); anything else a CTA-per-row kernel that
// re-reads the row from L2. Semantics follow the reference (see tfx.h):
// EXCLUDE restates the f32 attention rows of crates/cpu-kernels/src/lib.rs:
// 1053-1080, FILL the tenferro-infer masked_softmax (softmax.rs:26-34,
// util.rs:87).
//
// The analytic mask conditions (valid length, causality, sliding window) all
// keep one interval of keys per row, so each row computes [lo, hi) once and
// every key is tested with one unsigned compare. The division p = e / sum is
// done as e * (1/sum) followed by one FMA correction step (Markstein), which
// returns the correctly rounded quotient for normal results; a row with a
// numerator that could produce a subnormal quotient takes the IEEE division.

#include <cmath>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace tfx {
namespace {

struct MaskArgs {
  int64_t heads, q_len, k_len;
  int64_t row_offset;  // global index of the first row handed to the kernel
  int64_t window, valid_len;
  const int32_t* valid_lens;
  const float* add;
  int64_t add_sb, add_sq, add_sk;
  const uint8_t* keep;
  int64_t keep_sb, keep_sq, keep_sk;
  float scale;
  int causal, skip_invalid_q;
  // Rows < 2^32 (always, below): q = row mod q_len and b = row / (heads*q_len)
  // by 32-bit multiply-shift division instead of 64-bit division.
  bool rows32;
  FastDiv div_q, div_bq;
};

// Keys [lo, lo + span) of a row pass the analytic conditions.
struct RowCtx {
  int64_t b, q;
  uint32_t lo, span;  // kept iff (uint32)(k - lo) < span
};

__device__ __forceinline__ RowCtx row_ctx(const MaskArgs& m, uint64_t local_row) {
  RowCtx c;
  const uint64_t row = local_row + uint64_t(m.row_offset);
  if (m.rows32) {
    const uint32_t r32 = uint32_t(row);
    c.q = int64_t(r32 - m.div_q.div(r32) * m.div_q.d);
    c.b = int64_t(m.div_bq.div(r32));
  } else {
    c.q = int64_t(row % uint64_t(m.q_len));
    c.b = int64_t(row / uint64_t(m.heads * m.q_len));
  }
  const int64_t vlen = m.valid_lens ? int64_t(m.valid_lens[c.b]) : m.valid_len;
  int64_t lo = 0, hi = m.k_len;
  if (vlen >= 0) hi = min(hi, vlen);
  if (m.causal) hi = min(hi, c.q + 1);
  if (m.window >= 0 && !(m.skip_invalid_q && vlen >= 0 && c.q >= vlen)) {
    lo = max(lo, c.q - m.window);
    hi = min(hi, c.q + m.window + 1);
  }
  if (hi < lo) hi = lo;
  c.lo = uint32_t(lo);
  c.span = uint32_t(hi - lo);
  return c;
}

constexpr int kExclude = TFX_SOFTMAX_EXCLUDE;

// Masked, scaled score of key k (in range). EXCLUDE: -inf when masked;
// FILL: -1e30 when masked (util.rs:87).
template <int SEM, bool TENSORS>
__device__ __forceinline__ float score(const MaskArgs& m, const RowCtx& c, uint32_t k, float s) {
  bool keep = k - c.lo < c.span;
  if constexpr (TENSORS) {
    if (m.keep && m.keep[c.b * m.keep_sb + c.q * m.keep_sq + int64_t(k) * m.keep_sk] == 0)
      keep = false;
  }
  float v = __fmul_rn(s, m.scale);
  if constexpr (TENSORS) {
    if (m.add && keep)
      v = __fadd_rn(v, __ldg(m.add + c.b * m.add_sb + c.q * m.add_sq + int64_t(k) * m.add_sk));
  }
  return keep ? v : (SEM == kExclude ? -INFINITY : -1.0e30f);
}

// exp(v - max); EXCLUDE: non-finite v (masked, NaN, inf) contributes 0.
template <int SEM>
__device__ __forceinline__ float expo(float v, float mx) {
  const float e = expf(__fsub_rn(v, mx));
  if constexpr (SEM == kExclude) return fabsf(v) < INFINITY ? e : 0.0f;
  return e;
}

// e / sum, correctly rounded (see the file comment); r = 1/sum rounded.
__device__ __forceinline__ float quotient(float e, float sum, float r, bool fast) {
  float q = __fmul_rn(e, r);
  if (fast && e >= 0x1p-100f) {
    const float res = __fmaf_rn(-q, sum, e);
    q = __fmaf_rn(res, r, q);
  } else if (e != 0.0f) {
    q = __fdiv_rn(e, sum);
  }
  return q;
}

// ---- one row, compacted onto the keys its mask can keep ---------------------------
//
// The threads of a row (a warp, or a CTA for long rows) take the float4 chunks
// that meet the row's kept interval [lo, lo + span) -- chunk c0 + t + STRIDE*j
// for thread t -- so reading, exp and division scale with the kept keys, not
// with k_len. Every key outside those chunks is masked: its probability is one
// per-row value p_out (0; NaN for an all-masked EXCLUDE row, 1/k_len for an
// all-masked FILL row), written without reading its score.

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  v = is_max ? warp_max(v) : warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = is_max ? -INFINITY : 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) r = is_max ? fmaxf(r, red[i]) : __fadd_rn(r, red[i]);
  return r;
}

// BAND: the row's kept chunks number at most NV * STRIDE (guaranteed by the
// caller from the analytic mask) while kv may be larger; the masked rest is
// written by a loop over the whole row. Otherwise kv <= NV * STRIDE.
template <int NV, int STRIDE, int SEM, bool TENSORS, bool BAND, class RMax, class RSum,
          class RAny>
__device__ __forceinline__ void softmax_row(const float4* __restrict__ src, float4* dst,
                                            const MaskArgs& m, const RowCtx& c, uint32_t kv,
                                            uint32_t tid, RMax rmax, RSum rsum, RAny rany) {
  constexpr float kMasked = SEM == kExclude ? -INFINITY : -1.0e30f;
  const uint32_t c0 = c.lo >> 2;
  const uint32_t hi = c.lo + c.span;
  const uint32_t nch = c.span ? ((hi - 1) >> 2) - c0 + 1 : 0;
  const bool scaled = m.scale != 1.0f;
  float v[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t idx = j * STRIDE + tid;
    if (idx < nch) {
      const float4 t = ld_stream(src + c0 + idx);
      v[j][0] = t.x; v[j][1] = t.y; v[j][2] = t.z; v[j][3] = t.w;
    }
  }
  // Scale and mask. Chunks inside [lo, hi) need no per-key test.
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (j * STRIDE < nch) {  // uniform over the row's threads
      const uint32_t idx = j * STRIDE + tid;
      if (idx < nch) {
        const uint32_t k0 = (c0 + idx) << 2;
        if constexpr (TENSORS) {
#pragma unroll
          for (int e = 0; e < 4; ++e) v[j][e] = score<SEM, true>(m, c, k0 + e, v[j][e]);
        } else {
          if (scaled) {
            const float2 sc = make_float2(m.scale, m.scale);
            const float2 a = __fmul2_rn(make_float2(v[j][0], v[j][1]), sc);
            const float2 b = __fmul2_rn(make_float2(v[j][2], v[j][3]), sc);
            v[j][0] = a.x; v[j][1] = a.y; v[j][2] = b.x; v[j][3] = b.y;
          }
          if (k0 < c.lo || k0 + 4 > hi) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (k0 + e - c.lo >= c.span) v[j][e] = kMasked;
          }
        }
        mx = fmaxf(mx, fmaxf(fmaxf(v[j][0], v[j][1]), fmaxf(v[j][2], v[j][3])));
      }
    }
  }
  // FILL: the keys outside the processed chunks hold -1e30 as well.
  if (SEM != kExclude && nch < kv) mx = fmaxf(mx, -1.0e30f);
  mx = rmax(mx);
  // exp(v - max). EXCLUDE: a non-finite score (masked -inf, NaN, +inf) must
  // contribute 0; every such case makes exp return NaN or 0 here, and
  // fmaxf(e, 0) maps NaN to 0 and leaves every other e >= 0 unchanged.
  float2 acc = make_float2(0.0f, 0.0f);
  bool tiny = false;  // a nonzero e < 2^-100: its quotient could be subnormal
  const float2 nmx = make_float2(-mx, -mx);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (j * STRIDE < nch) {
      const uint32_t idx = j * STRIDE + tid;
      if (idx < nch) {
        const float2 d0 = __fadd2_rn(make_float2(v[j][0], v[j][1]), nmx);
        const float2 d1 = __fadd2_rn(make_float2(v[j][2], v[j][3]), nmx);
        float e0 = expf(d0.x), e1 = expf(d0.y), e2 = expf(d1.x), e3 = expf(d1.y);
        if constexpr (SEM == kExclude) {
          e0 = fmaxf(e0, 0.0f); e1 = fmaxf(e1, 0.0f); e2 = fmaxf(e2, 0.0f); e3 = fmaxf(e3, 0.0f);
        }
        v[j][0] = e0; v[j][1] = e1; v[j][2] = e2; v[j][3] = e3;
        acc = __fadd2_rn(acc, make_float2(e0, e1));
        acc = __fadd2_rn(acc, make_float2(e2, e3));
        // bits(e) - 1 < bits(2^-100) - 1 (unsigned)  <=>  0 < e < 2^-100
        const uint32_t lim = 0x0D800000u - 1u;
        const uint32_t b = min(min(__float_as_uint(e0) - 1u, __float_as_uint(e1) - 1u),
                               min(__float_as_uint(e2) - 1u, __float_as_uint(e3) - 1u));
        tiny |= b < lim;
      }
    }
  }
  float sum = rsum(__fadd_rn(acc.x, acc.y));
  // exp of a key outside the processed chunks: 0, or 1 when the whole FILL row
  // is masked (then every one of them adds 1, as the dense sum would).
  float e_out = 0.0f;
  if (SEM != kExclude && nch < kv) {
    e_out = expf(__fsub_rn(-1.0e30f, mx));
    sum = __fadd_rn(sum, __fmul_rn(float(4 * (kv - nch)), e_out));
  }
  const float r = __frcp_rn(sum);
  // Quotients e * (1/sum) + one FMA correction: correctly rounded when the
  // result is normal (sum < 2^24, e == 0 or e >= 2^-100); otherwise every
  // element of the row takes the IEEE division.
  const bool slow = rany(tiny || !(sum < 0x1p24f));
  const float2 r2 = make_float2(r, r), ns2 = make_float2(-sum, -sum);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (j * STRIDE < nch) {
      const uint32_t idx = j * STRIDE + tid;
      if (idx < nch) {
        float4 o;
        if (!slow) {
          const float2 a = make_float2(v[j][0], v[j][1]), b = make_float2(v[j][2], v[j][3]);
          float2 qa = __fmul2_rn(a, r2), qb = __fmul2_rn(b, r2);
          qa = __ffma2_rn(__ffma2_rn(qa, ns2, a), r2, qa);
          qb = __ffma2_rn(__ffma2_rn(qb, ns2, b), r2, qb);
          o = make_float4(qa.x, qa.y, qb.x, qb.y);
        } else {
          o = make_float4(__fdiv_rn(v[j][0], sum), __fdiv_rn(v[j][1], sum),
                          __fdiv_rn(v[j][2], sum), __fdiv_rn(v[j][3], sum));
        }
        dst[c0 + idx] = o;
      }
    }
  }
  if (nch < kv) {  // uniform over the row's threads
    const float p_out = __fdiv_rn(e_out, sum);
    const float4 fill = make_float4(p_out, p_out, p_out, p_out);
    if constexpr (BAND) {
      for (uint32_t q4 = tid; q4 < kv; q4 += STRIDE)
        if (q4 - c0 >= nch) dst[q4] = fill;
    } else {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const uint32_t q4 = j * STRIDE + tid;
        if (q4 < kv && q4 - c0 >= nch) dst[q4] = fill;
      }
    }
  }
}

// ---- LANES (8, 16 or 32) threads per row (k_len <= 1024) ---------------------------
//
// Short rows are shared by fewer threads so that each thread holds up to 32
// keys: the per-row work (index decomposition, interval, reductions, the
// reciprocal) is then spread over more keys. 256 / LANES rows per CTA; the
// shuffles of a row stay inside its aligned group of LANES lanes.

template <int LANES>
__device__ __forceinline__ float group_max(float v, unsigned mask) {
#pragma unroll
  for (int d = LANES / 2; d >= 1; d >>= 1) v = fmaxf(v, __shfl_xor_sync(mask, v, d));
  return v;
}
template <int LANES>
__device__ __forceinline__ float group_sum(float v, unsigned mask) {
#pragma unroll
  for (int d = LANES / 2; d >= 1; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(mask, v, d));
  return v;
}

template <int NV, int LANES, int SEM, bool TENSORS, bool BAND = false>
__global__ void __launch_bounds__(256) softmax_lanes_kernel(const float* __restrict__ s,
                                                            float* __restrict__ p, uint64_t rows,
                                                            MaskArgs m) {
  static_assert(LANES == 8 || LANES == 16 || LANES == 32, "LANES");
  pdl_enter();
  const uint32_t lane = threadIdx.x & (LANES - 1);
  const uint64_t row = uint64_t(blockIdx.x) * (256 / LANES) + threadIdx.x / LANES;
  if (row >= rows) return;  // the row's whole group leaves together
  const unsigned mask =
      LANES == 32 ? 0xffffffffu : ((1u << LANES) - 1u) << (threadIdx.x & 31 & ~(LANES - 1));
  const RowCtx c = row_ctx(m, row);
  const uint32_t kv = uint32_t(m.k_len / 4);
  softmax_row<NV, LANES, SEM, TENSORS, BAND>(
      reinterpret_cast<const float4*>(s + row * uint64_t(m.k_len)),
      reinterpret_cast<float4*>(p + row * uint64_t(m.k_len)), m, c, kv, lane,
      [mask](float x) { return group_max<LANES>(x, mask); },
      [mask](float x) { return group_sum<LANES>(x, mask); },
      [mask](bool b) { return __any_sync(mask, b) != 0; });
}

// ---- CTA (256 threads) per row (k_len <= 8192) -------------------------------------

template <int NV, int SEM, bool TENSORS>
__global__ void __launch_bounds__(256) softmax_cta_kernel(const float* __restrict__ s,
                                                          float* __restrict__ p, MaskArgs m) {
  pdl_enter();
  __shared__ float red[8];
  const uint64_t row = blockIdx.x;
  const RowCtx c = row_ctx(m, row);
  const uint32_t kv = uint32_t(m.k_len / 4);
  softmax_row<NV, 256, SEM, TENSORS, false>(
      reinterpret_cast<const float4*>(s + row * uint64_t(m.k_len)),
      reinterpret_cast<float4*>(p + row * uint64_t(m.k_len)), m, c, kv, threadIdx.x,
      [&](float x) { return block_reduce(x, red, true); },
      [&](float x) { return block_reduce(x, red, false); },
      [](bool b) { return __syncthreads_or(b) != 0; });
}

// ---- any length / alignment: CTA per row, three passes (row re-read from L2) ----

template <int SEM, bool TENSORS>
__global__ void __launch_bounds__(256) softmax_generic_kernel(const float* s, float* p,
                                                              MaskArgs m) {
  pdl_enter();
  __shared__ float red[8];
  const uint64_t row = blockIdx.x;
  const RowCtx c = row_ctx(m, row);
  const float* src = s + row * uint64_t(m.k_len);
  float* dst = p + row * uint64_t(m.k_len);
  const uint32_t n = uint32_t(m.k_len);
  // Scores outside the row's analytic interval are never read: they cannot
  // reach the result (masked keys are -inf / -1e30 whatever they hold).
  auto at = [&](uint32_t k) { return k - c.lo < c.span ? src[k] : 0.0f; };
  float mx = -INFINITY;
  for (uint32_t k = threadIdx.x; k < n; k += 256)
    mx = fmaxf(mx, score<SEM, TENSORS>(m, c, k, at(k)));
  mx = block_reduce(mx, red, true);
  float sum = 0.0f;
  for (uint32_t k = threadIdx.x; k < n; k += 256)
    sum = __fadd_rn(sum, expo<SEM>(score<SEM, TENSORS>(m, c, k, at(k)), mx));
  sum = block_reduce(sum, red, false);
  const float r = __frcp_rn(sum);
  const bool fast = sum < 0x1p24f;
  // In place (dst == src) each thread reads, then writes, only its own keys.
  for (uint32_t k = threadIdx.x; k < n; k += 256)
    dst[k] = quotient(expo<SEM>(score<SEM, TENSORS>(m, c, k, at(k)), mx), sum, r, fast);
}

template <int SEM, bool TENSORS>
int launch_softmax(const char* op, const float* scores, float* probs, int64_t rows, int64_t kl,
                   const MaskArgs& m, cudaStream_t stream) {
  const bool vec = kl % 4 == 0 && aligned(scores, 16) && aligned(probs, 16);
  const int64_t kv = kl / 4;
  // A sliding window bounds every row's kept interval to 2 * window + 1
  // keys: eight lanes per row hold the band (at most 40 chunks, five per
  // lane) and write the masked rest of the row in a loop, so the per-row work
  // is spread over 8 lanes whatever k_len is.
  // (Not when padded queries drop the window: their interval is the whole
  // valid prefix.)
  const int64_t band_chunks = m.window >= 0 ? (2 * m.window + 1 + 3) / 4 + 1 : kv;
  if (!TENSORS && vec && m.window >= 0 && !m.skip_invalid_q && band_chunks <= 8 * 5 &&
      kv > 8 * 5) {
    const int64_t per = 32;
    TFX_REQUIRE(rows / per < (int64_t(1) << 31), op, "shape", "too many rows for one call");
    return launch_kernel(op, softmax_lanes_kernel<5, 8, SEM, TENSORS, true>,
                         dim3(unsigned((rows + per - 1) / per)), dim3(256), 0, stream, 1, scores,
                         probs, uint64_t(rows), m);
  }
  if (vec && kv <= 32 * 8) {
    // Up to 32 keys per thread: 8 lanes per row up to 256 keys, 16 up to
    // 512, a warp up to 1024.
#define TFX_SM_LANES(NV, LANES)                                                           \
  if (kv <= LANES * NV) {                                                                 \
    const int64_t per = 256 / LANES;                                                      \
    TFX_REQUIRE(rows / per < (int64_t(1) << 31), op, "shape", "too many rows for one call"); \
    return launch_kernel(op, softmax_lanes_kernel<NV, LANES, SEM, TENSORS>,                 \
                         dim3(unsigned((rows + per - 1) / per)), dim3(256), 0, stream, 1,   \
                         scores, probs, uint64_t(rows), m);                                 \
  }
    TFX_SM_LANES(1, 8)
    TFX_SM_LANES(2, 8)
    TFX_SM_LANES(4, 8)
    TFX_SM_LANES(8, 8)
    TFX_SM_LANES(6, 16)
    TFX_SM_LANES(8, 16)
    TFX_SM_LANES(6, 32)
    TFX_SM_LANES(8, 32)
#undef TFX_SM_LANES
  }
  TFX_REQUIRE(rows < (int64_t(1) << 31), op, "shape", "too many rows for one call");
  const unsigned grid = unsigned(rows);
  if (vec && kv <= 256 * 8) {
#define TFX_SM_CTA(NV)                                                              \
  if (kv <= 256 * NV) {                                                             \
    return launch_kernel(op, softmax_cta_kernel<NV, SEM, TENSORS>, dim3(grid), dim3(256), 0, \
                         stream, 1, scores, probs, m);                                         \
  }
    TFX_SM_CTA(2)
    TFX_SM_CTA(4)
    TFX_SM_CTA(8)
#undef TFX_SM_CTA
  }
  return launch_kernel(op, softmax_generic_kernel<SEM, TENSORS>, dim3(grid), dim3(256), 0, stream,
                       1, scores, probs, m);
}

}  // namespace

// Rows [row_begin, row_begin + row_count) of the softmax described by d;
// scores / probs point at row row_begin. Arguments are validated by the caller.
int masked_softmax_rows(const float* scores, float* probs, const tfx_softmax_desc* d,
                        int64_t row_begin, int64_t row_count, cudaStream_t stream) {
  const char* op = "tenferro-infer::masked_softmax";
  if (row_count == 0) return TFX_OK;
  MaskArgs m;
  m.row_offset = row_begin;
  const int64_t total_rows = d->batch * d->heads * d->q_len;
  m.rows32 = total_rows < (int64_t(1) << 31) && d->heads * d->q_len < (int64_t(1) << 31);
  if (m.rows32) {
    m.div_q = FastDiv(uint32_t(d->q_len));
    m.div_bq = FastDiv(uint32_t(d->heads * d->q_len));
  }
  m.heads = d->heads;
  m.q_len = d->q_len;
  m.k_len = d->k_len;
  m.window = d->window;
  m.valid_len = d->valid_len;
  m.valid_lens = d->valid_lens;
  m.add = d->add_mask;
  m.add_sb = d->add_stride_b;
  m.add_sq = d->add_stride_q;
  m.add_sk = d->add_stride_k;
  m.keep = d->keep;
  m.keep_sb = d->keep_stride_b;
  m.keep_sq = d->keep_stride_q;
  m.keep_sk = d->keep_stride_k;
  m.scale = d->scale;
  m.causal = d->causal ? 1 : 0;
  m.skip_invalid_q = d->window_skips_invalid_query ? 1 : 0;
  const bool tensors = m.add != nullptr || m.keep != nullptr;
  const int64_t kl = d->k_len;
  if (d->semantics == TFX_SOFTMAX_EXCLUDE) {
    if (tensors) return launch_softmax<TFX_SOFTMAX_EXCLUDE, true>(op, scores, probs, row_count, kl, m, stream);
    return launch_softmax<TFX_SOFTMAX_EXCLUDE, false>(op, scores, probs, row_count, kl, m, stream);
  }
  if (tensors) return launch_softmax<TFX_SOFTMAX_FILL, true>(op, scores, probs, row_count, kl, m, stream);
  return launch_softmax<TFX_SOFTMAX_FILL, false>(op, scores, probs, row_count, kl, m, stream);
}

int validate_softmax(const float* scores, const float* probs, const tfx_softmax_desc* d,
                     int64_t* rows_out) {
  const char* op = "tenferro-infer::masked_softmax";
  TFX_REQUIRE(d, op, "desc", "null pointer");
  TFX_REQUIRE(d->batch >= 0 && d->heads >= 0 && d->q_len >= 0 && d->k_len >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(d->semantics == TFX_SOFTMAX_EXCLUDE || d->semantics == TFX_SOFTMAX_FILL, op,
              "semantics", "unknown semantics " + std::to_string(d->semantics));
  TFX_REQUIRE(d->k_len < (int64_t(1) << 31), op, "k_len", "rows longer than 2^31 keys");
  const int64_t rows = d->batch * d->heads * d->q_len;
  *rows_out = d->k_len == 0 ? 0 : rows;
  if (rows == 0 || d->k_len == 0) return TFX_OK;
  TFX_REQUIRE(scores && probs, op, scores ? "probs" : "scores", "null pointer");
  const size_t bytes = size_t(rows) * size_t(d->k_len) * 4;
  TFX_REQUIRE(probs == scores || !overlaps(scores, bytes, probs, bytes), op, "probs",
              "partially overlaps scores");
  TFX_REQUIRE(rows < (int64_t(1) << 40), op, "shape", "too many rows");
  return TFX_OK;
}

}  // namespace tfx

using namespace tfx;

extern "C" int tfx_masked_softmax_f32(const float* scores, float* probs,
                                      const tfx_softmax_desc* d, tfx_stream_t stream) {
  clear_error();
  int64_t rows = 0;
  int rc = validate_softmax(scores, probs, d, &rows);
  if (rc != TFX_OK || rows == 0) return rc;
  device_info(&rc);
  if (rc != TFX_OK) return rc;
  return masked_softmax_rows(scores, probs, d, 0, rows, stream);
}
