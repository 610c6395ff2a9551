// softmax.cu -- masked row softmax over row-major [batch][heads][q_len][k_len]
// scores (keys contiguous).
//
// One warp owns one row of up to 1024 keys: the row is read once with 128-bit
// loads into registers, the mask is evaluated from (q, k) arithmetic (window,
// valid length, causality) plus the optional additive / boolean mask tensors,
// the max and the sum are warp-shuffle reductions over registers, and the
// probabilities are written once. Longer rows use a CTA per row (up to 8192
// keys in registers); anything else a CTA-per-row kernel that re-reads the row
// from L2. Semantics follow the reference (see tfx.h): EXCLUDE restates the
// f32 attention rows of crates/cpu-kernels/src/lib.rs:1053-1080, FILL the
// tenferro-infer masked_softmax (softmax.rs:26-34, util.rs:87).

#include <cmath>
#include <string>

#include "common.cuh"

namespace tfx {
namespace {

struct MaskArgs {
  int64_t heads, q_len, k_len;
  int64_t window, valid_len;
  const int32_t* valid_lens;
  const float* add;
  int64_t add_sb, add_sq, add_sk;
  const uint8_t* keep;
  int64_t keep_sb, keep_sq, keep_sk;
  float scale;
  int causal, skip_invalid_q, semantics;
};

struct RowCtx {
  int64_t b, q, vlen;
  bool window_on;
};

__device__ __forceinline__ RowCtx row_ctx(const MaskArgs& m, uint64_t row) {
  RowCtx c;
  c.q = int64_t(row % uint64_t(m.q_len));
  c.b = int64_t(row / uint64_t(m.heads * m.q_len));
  c.vlen = m.valid_lens ? int64_t(m.valid_lens[c.b]) : m.valid_len;
  c.window_on = m.window >= 0 && !(m.skip_invalid_q && c.vlen >= 0 && c.q >= c.vlen);
  return c;
}

template <bool TENSORS>
__device__ __forceinline__ bool kept(const MaskArgs& m, const RowCtx& c, int64_t k) {
  if (c.vlen >= 0 && k >= c.vlen) return false;
  if (m.causal && k > c.q) return false;
  if (c.window_on) {
    const int64_t diff = c.q > k ? c.q - k : k - c.q;
    if (diff > m.window) return false;
  }
  if constexpr (TENSORS) {
    if (m.keep && m.keep[c.b * m.keep_sb + c.q * m.keep_sq + k * m.keep_sk] == 0) return false;
  }
  return true;
}

// The masked, scaled score of key k (EXCLUDE: -inf when masked; FILL: -1e30).
template <bool TENSORS>
__device__ __forceinline__ float score(const MaskArgs& m, const RowCtx& c, int64_t k, float s) {
  const bool keep = kept<TENSORS>(m, c, k);
  if (m.semantics == TFX_SOFTMAX_EXCLUDE && !keep) return -INFINITY;
  float v = __fmul_rn(s, m.scale);
  if constexpr (TENSORS) {
    if (m.add) v = __fadd_rn(v, __ldg(m.add + c.b * m.add_sb + c.q * m.add_sq + k * m.add_sk));
  }
  if (!keep) v = -1.0e30f;
  return v;
}

// p = exp(v - max), EXCLUDE: non-finite v contributes 0.
__device__ __forceinline__ float expo(const MaskArgs& m, float v, float mx) {
  if (m.semantics == TFX_SOFTMAX_EXCLUDE && !isfinite(v)) return 0.0f;
  return expf(__fsub_rn(v, mx));
}

// ---- warp per row, NV float4 per lane ------------------------------------------

template <int NV, bool TENSORS>
__global__ void __launch_bounds__(256) softmax_warp_kernel(const float* __restrict__ s,
                                                           float* __restrict__ p, uint64_t rows,
                                                           MaskArgs m) {
  const int lane = threadIdx.x & 31;
  const uint64_t row = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;  // the whole warp leaves together
  const RowCtx c = row_ctx(m, row);
  const uint32_t kv = uint32_t(m.k_len / 4);
  const float4* src = reinterpret_cast<const float4*>(s + row * uint64_t(m.k_len));
  float v[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 32 + lane;
    if (q4 < kv) {
      const float4 t = ld_stream(src + q4);
      v[j][0] = t.x; v[j][1] = t.y; v[j][2] = t.z; v[j][3] = t.w;
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 32 + lane;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[j][e] = q4 < kv ? score<TENSORS>(m, c, int64_t(q4) * 4 + e, v[j][e]) : -INFINITY;
      mx = fmaxf(mx, v[j][e]);
    }
  }
  mx = warp_max(mx);
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 32 + lane;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[j][e] = q4 < kv ? expo(m, v[j][e], mx) : 0.0f;
      sum = __fadd_rn(sum, v[j][e]);
    }
  }
  sum = warp_sum(sum);
  float4* dst = reinterpret_cast<float4*>(p + row * uint64_t(m.k_len));
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 32 + lane;
    if (q4 < kv)
      dst[q4] = make_float4(__fdiv_rn(v[j][0], sum), __fdiv_rn(v[j][1], sum),
                            __fdiv_rn(v[j][2], sum), __fdiv_rn(v[j][3], sum));
  }
}

// ---- CTA (256 threads) per row, NV float4 per thread ----------------------------

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

template <int NV, bool TENSORS>
__global__ void __launch_bounds__(256) softmax_cta_kernel(const float* __restrict__ s,
                                                          float* __restrict__ p, MaskArgs m) {
  __shared__ float red[8];
  const uint64_t row = blockIdx.x;
  const RowCtx c = row_ctx(m, row);
  const uint32_t kv = uint32_t(m.k_len / 4);
  const float4* src = reinterpret_cast<const float4*>(s + row * uint64_t(m.k_len));
  float v[NV][4];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 256 + threadIdx.x;
    if (q4 < kv) {
      const float4 t = ld_stream(src + q4);
      v[j][0] = t.x; v[j][1] = t.y; v[j][2] = t.z; v[j][3] = t.w;
    }
  }
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 256 + threadIdx.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[j][e] = q4 < kv ? score<TENSORS>(m, c, int64_t(q4) * 4 + e, v[j][e]) : -INFINITY;
      mx = fmaxf(mx, v[j][e]);
    }
  }
  mx = block_reduce(mx, red, true);
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 256 + threadIdx.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[j][e] = q4 < kv ? expo(m, v[j][e], mx) : 0.0f;
      sum = __fadd_rn(sum, v[j][e]);
    }
  }
  sum = block_reduce(sum, red, false);
  float4* dst = reinterpret_cast<float4*>(p + row * uint64_t(m.k_len));
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q4 = j * 256 + threadIdx.x;
    if (q4 < kv)
      dst[q4] = make_float4(__fdiv_rn(v[j][0], sum), __fdiv_rn(v[j][1], sum),
                            __fdiv_rn(v[j][2], sum), __fdiv_rn(v[j][3], sum));
  }
}

// ---- any length / alignment: CTA per row, three passes (row re-read from L2) ----

template <bool TENSORS>
__global__ void __launch_bounds__(256) softmax_generic_kernel(const float* s, float* p,
                                                              MaskArgs m) {
  __shared__ float red[8];
  const uint64_t row = blockIdx.x;
  const RowCtx c = row_ctx(m, row);
  const float* src = s + row * uint64_t(m.k_len);
  float* dst = p + row * uint64_t(m.k_len);
  float mx = -INFINITY;
  for (int64_t k = threadIdx.x; k < m.k_len; k += 256) mx = fmaxf(mx, score<TENSORS>(m, c, k, src[k]));
  mx = block_reduce(mx, red, true);
  float sum = 0.0f;
  for (int64_t k = threadIdx.x; k < m.k_len; k += 256)
    sum = __fadd_rn(sum, expo(m, score<TENSORS>(m, c, k, src[k]), mx));
  sum = block_reduce(sum, red, false);
  __syncthreads();  // every read of src precedes any write of dst (in-place calls)
  // In place, dst == src: each thread reads then writes only its own keys.
  for (int64_t k = threadIdx.x; k < m.k_len; k += 256)
    dst[k] = __fdiv_rn(expo(m, score<TENSORS>(m, c, k, src[k]), mx), sum);
}

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" int tfx_masked_softmax_f32(const float* scores, float* probs,
                                      const tfx_softmax_desc* d, tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-infer::masked_softmax";
  TFX_REQUIRE(d, op, "desc", "null pointer");
  TFX_REQUIRE(d->batch >= 0 && d->heads >= 0 && d->q_len >= 0 && d->k_len >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(d->semantics == TFX_SOFTMAX_EXCLUDE || d->semantics == TFX_SOFTMAX_FILL, op,
              "semantics", "unknown semantics " + std::to_string(d->semantics));
  const int64_t rows = d->batch * d->heads * d->q_len;
  if (rows == 0 || d->k_len == 0) return TFX_OK;
  TFX_REQUIRE(scores && probs, op, scores ? "probs" : "scores", "null pointer");
  const size_t bytes = size_t(rows) * size_t(d->k_len) * 4;
  TFX_REQUIRE(probs == scores || !overlaps(scores, bytes, probs, bytes), op, "probs",
              "partially overlaps scores");
  TFX_REQUIRE(rows < (int64_t(1) << 40), op, "shape", "too many rows");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;

  MaskArgs m;
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
  m.semantics = d->semantics;
  const bool tensors = m.add != nullptr || m.keep != nullptr;

  const bool vec = d->k_len % 4 == 0 && aligned(scores, 16) && aligned(probs, 16);
  const int64_t kv = d->k_len / 4;
  if (vec && kv <= 32 * 8) {
    TFX_REQUIRE(rows / 8 < (int64_t(1) << 31), op, "shape", "too many rows for one call");
    const unsigned grid = unsigned((rows + 7) / 8);
#define TFX_SM_WARP(NV)                                                                       \
  if (kv <= 32 * NV) {                                                                        \
    if (tensors) softmax_warp_kernel<NV, true><<<grid, 256, 0, stream>>>(scores, probs, rows, m); \
    else softmax_warp_kernel<NV, false><<<grid, 256, 0, stream>>>(scores, probs, rows, m);   \
    return check_launch(op);                                                                  \
  }
    TFX_SM_WARP(1)
    TFX_SM_WARP(2)
    TFX_SM_WARP(3)
    TFX_SM_WARP(4)
    TFX_SM_WARP(6)
    TFX_SM_WARP(8)
#undef TFX_SM_WARP
  }
  TFX_REQUIRE(rows < (int64_t(1) << 31), op, "shape", "too many rows for one call");
  const unsigned grid = unsigned(rows);
  if (vec && kv <= 256 * 8) {
#define TFX_SM_CTA(NV)                                                                   \
  if (kv <= 256 * NV) {                                                                  \
    if (tensors) softmax_cta_kernel<NV, true><<<grid, 256, 0, stream>>>(scores, probs, m); \
    else softmax_cta_kernel<NV, false><<<grid, 256, 0, stream>>>(scores, probs, m);     \
    return check_launch(op);                                                             \
  }
    TFX_SM_CTA(2)
    TFX_SM_CTA(4)
    TFX_SM_CTA(8)
#undef TFX_SM_CTA
  }
  if (tensors) softmax_generic_kernel<true><<<grid, 256, 0, stream>>>(scores, probs, m);
  else softmax_generic_kernel<false><<<grid, 256, 0, stream>>>(scores, probs, m);
  return check_launch(op);
}
