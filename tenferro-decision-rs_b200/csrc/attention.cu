// attention.cu -- the attention cores of the Laya (ModernBERT) and Jeff
// (Qwen3.5) forwards: the prep kernels that bring q, k, v into head-major
// (batch, heads, length, head_dim) form, and masked scaled dot-product
// attention over head-major tensors.
//
// The reference's CUDA path has the same two stages (fused_laya_qkv_prep /
// fused_jeff_qkv_prep, then fused_attention, crates/tenferro-ext/src/cuda/
// fused.cu:150-306, driven by FusedScope, cuda_fused.rs:751-1103); its CPU ops
// fix the arithmetic (crates/cpu-kernels/src/lib.rs:618-760 Jeff,
// :819-1150 Laya). The prep kernels reproduce that arithmetic bit for bit
// (rounded products, sequential per-token sums). The attention kernel is a
// tiled online-softmax ("flash") kernel on the f32 pipes: a CTA owns 64
// queries of one head, streams 64-key blocks of K and V through shared
// memory, keeps the running max, sum and the 64 x head_dim output tile in
// registers, and skips key blocks that the mask excludes entirely.

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"
#include "tma.cuh"

namespace tfx {
namespace {

// ---- tile images ------------------------------------------------------------------------
//
// The tensor-core attention (head_dim 64) reads q, k and v as tf32 hi / lo
// "tile images": byte for byte the shared-memory layout its MMAs read (layout
// described in attn_ws.cuh), written once by the Laya prep kernel or by
// attn_img_split_kernel. Per head: Q in 128-query tiles (hi 32 KB then lo
// 32 KB), K and V in 64-key tiles (hi 16 KB then lo 16 KB each).
constexpr int kWsTQ = 128;                  // queries per tile
constexpr int kWsKB = 64;                   // keys per tile
constexpr uint32_t kWsQRegion = 16384;      // 128 rows x 128 bytes
constexpr uint32_t kWsKRegion = 8192;       // 64 rows x 128 bytes
constexpr uint32_t kWsQPlane = 2 * kWsQRegion;   // Q hi or Q lo
constexpr uint32_t kWsTile = 2 * kWsKRegion;     // K / V hi or lo
constexpr uint32_t kWsSlot = 2 * kWsTile;        // hi + lo

// Byte offsets inside the tile images (and inside the shared-memory copies
// of the tiles), for 4 consecutive channels ch .. ch + 3 (ch % 4 == 0) of
// row r of the tile.
__host__ __device__ __forceinline__ uint32_t img_kmajor_off(uint32_t r, uint32_t ch,
                                                            uint32_t region_bytes) {
  return (ch >> 5) * region_bytes + r * 128 + ((((ch & 31) >> 2) ^ (r & 7)) << 4);
}
__host__ __device__ __forceinline__ uint32_t img_v_off(uint32_t r, uint32_t ch) {
  return (ch >> 5) * kWsKRegion + r * 128 + ((((ch & 31) >> 3) ^ (r & 3)) << 5) +
         (((ch & 7) >> 2) << 4);
}

// hi / lo of 4 values for a tile image: hi = tf32(x), lo = x - hi (exact);
// a value the tensor cores cannot take (non-finite, or beyond the largest
// tf32) is kept whole in hi with lo = 0, so hi + lo gives back every value.
__device__ __forceinline__ void img_split4(float4 x, float4* hi, float4* lo, bool* bad) {
  constexpr float kMax = 3.4e38f;  // below the largest tf32 (rounding up stays finite)
  float h[4], l[4];
  const float v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool ok = fabsf(v[i]) < kMax;
    *bad |= !ok;
    h[i] = ok ? tf32_round_finite(v[i]) : v[i];
    l[i] = ok ? __fsub_rn(v[i], h[i]) : 0.0f;
  }
  *hi = make_float4(h[0], h[1], h[2], h[3]);
  *lo = make_float4(l[0], l[1], l[2], l[3]);
}


// ---- Laya prep: split + full-width RoPE ------------------------------------------------

// One thread per (token row, head, VEC pairs): q and k pairs (i, i + half)
// rotated as a*c - b*s, a*s + b*c with every product rounded (lib.rs:
// 996-1008); v copied. IMG (head_dim 64, VEC 4): q, k, v go straight into the
// tensor-core attention's tile images (qimg / kimg / vimg, nqt / nkt tiles
// per head) instead of the head-major qh / kh / vh. LATE: the grid waits for
// the previous one at its end instead of its start. The previous grid is then
// the mask digest, which waited for everything before it and let this grid
// start at once; this grid reads nothing the digest writes, and waiting at the
// end makes its completion imply the digest's for the attention that follows.
// LATE also lets the attention grid launch as soon as every CTA of this one
// has started (the attention waits for this grid's completion before it reads
// anything).
template <int VEC, bool IMG = false, bool LATE = false>
__global__ void __launch_bounds__(256) laya_prep_kernel(
    const float* __restrict__ qkv, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, float* __restrict__ qh, float* __restrict__ kh,
    float* __restrict__ vh, uint32_t hidden, uint32_t heads, uint32_t length, uint32_t hd,
    uint64_t total, FastDiv div_chunks, FastDiv div_heads, FastDiv div_len, uint8_t* flags,
    uint8_t* __restrict__ qimg, uint8_t* __restrict__ kimg, uint8_t* __restrict__ vimg,
    uint32_t nqt, uint32_t nkt) {
  if constexpr (!LATE) pdl_enter();
  if constexpr (LATE) pdl_launch_dependents();
  const uint32_t half = hd / 2;
  for (uint64_t n = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; n < total;
       n += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t n32 = uint32_t(n);  // total < 2^32 (checked on the host)
    const uint32_t rest = div_chunks.div(n32);
    const uint32_t i0 = (n32 - rest * div_chunks.d) * VEC;
    const uint32_t row = div_heads.div(rest);  // b * length + l
    const uint32_t head = rest - row * div_heads.d;
    const uint32_t b = div_len.div(row), l = row - b * div_len.d;
    const float* src = qkv + uint64_t(3) * hidden * row + uint64_t(head) * hd;
    const uint64_t dst = ((uint64_t(b) * heads + head) * length + l) * hd;
    float qa[VEC], qb[VEC], ka[VEC], kb[VEC], va[VEC], vb[VEC], c[VEC], s[VEC];
    if constexpr (VEC == 4) {
      auto ld4 = [](const float* p, float* o) {
        const float4 t = ld_stream(reinterpret_cast<const float4*>(p));
        o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
      };
      ld4(src + i0, qa); ld4(src + half + i0, qb);
      ld4(src + hidden + i0, ka); ld4(src + hidden + half + i0, kb);
      ld4(src + 2 * hidden + i0, va); ld4(src + 2 * hidden + half + i0, vb);
      if (cos_t) {
        const float4 tc = __ldg(reinterpret_cast<const float4*>(cos_t + uint64_t(l) * half + i0));
        const float4 ts = __ldg(reinterpret_cast<const float4*>(sin_t + uint64_t(l) * half + i0));
        c[0] = tc.x; c[1] = tc.y; c[2] = tc.z; c[3] = tc.w;
        s[0] = ts.x; s[1] = ts.y; s[2] = ts.z; s[3] = ts.w;
      }
    } else {
      qa[0] = src[i0]; qb[0] = src[half + i0];
      ka[0] = src[hidden + i0]; kb[0] = src[hidden + half + i0];
      va[0] = src[2 * hidden + i0]; vb[0] = src[2 * hidden + half + i0];
      if (cos_t) {
        c[0] = __ldg(cos_t + uint64_t(l) * half + i0);
        s[0] = __ldg(sin_t + uint64_t(l) * half + i0);
      }
    }
    if (cos_t) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float a0 = qa[j], b0 = qb[j];
        qa[j] = __fsub_rn(__fmul_rn(a0, c[j]), __fmul_rn(b0, s[j]));
        qb[j] = __fadd_rn(__fmul_rn(a0, s[j]), __fmul_rn(b0, c[j]));
        const float a1 = ka[j], b1 = kb[j];
        ka[j] = __fsub_rn(__fmul_rn(a1, c[j]), __fmul_rn(b1, s[j]));
        kb[j] = __fadd_rn(__fmul_rn(a1, s[j]), __fmul_rn(b1, c[j]));
      }
    }
    if constexpr (IMG) {
      static_assert(VEC == 4, "tile images take 4 channels at a time");
      const uint64_t bh = uint64_t(b) * heads + head;
      bool bad = false;
      auto put = [&](uint8_t* tile, uint32_t plane, uint32_t off, const float* v) {
        float4 h, lo;
        img_split4(make_float4(v[0], v[1], v[2], v[3]), &h, &lo, &bad);
        *reinterpret_cast<float4*>(tile + off) = h;
        *reinterpret_cast<float4*>(tile + plane + off) = lo;
      };
      uint8_t* qt = qimg + (bh * nqt + l / kWsTQ) * (2 * kWsQPlane);
      const uint32_t rq = l % kWsTQ, rk = l % kWsKB;
      put(qt, kWsQPlane, img_kmajor_off(rq, i0, kWsQRegion), qa);
      put(qt, kWsQPlane, img_kmajor_off(rq, half + i0, kWsQRegion), qb);
      const uint64_t kv = (bh * nkt + l / kWsKB) * kWsSlot;
      put(kimg + kv, kWsTile, img_kmajor_off(rk, i0, kWsKRegion), ka);
      put(kimg + kv, kWsTile, img_kmajor_off(rk, half + i0, kWsKRegion), kb);
      put(vimg + kv, kWsTile, img_v_off(rk, i0), va);
      put(vimg + kv, kWsTile, img_v_off(rk, half + i0), vb);
      if (bad && flags) flags[bh] = 1;
      continue;
    }
    if (flags) {  // heads holding a value the tensor-core attention cannot take
      constexpr float kMax = 3.4e38f;
      bool bad = false;
#pragma unroll
      for (int j = 0; j < VEC; ++j)
        bad |= !(fabsf(qa[j]) < kMax && fabsf(qb[j]) < kMax && fabsf(ka[j]) < kMax &&
                 fabsf(kb[j]) < kMax && fabsf(va[j]) < kMax && fabsf(vb[j]) < kMax);
      if (bad) flags[b * heads + head] = 1;
    }
    if constexpr (VEC == 4) {
      auto st4 = [](float* p, const float* v) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
      };
      st4(qh + dst + i0, qa); st4(qh + dst + half + i0, qb);
      st4(kh + dst + i0, ka); st4(kh + dst + half + i0, kb);
      st4(vh + dst + i0, va); st4(vh + dst + half + i0, vb);
    } else {
      qh[dst + i0] = qa[0]; qh[dst + half + i0] = qb[0];
      kh[dst + i0] = ka[0]; kh[dst + half + i0] = kb[0];
      vh[dst + i0] = va[0]; vh[dst + half + i0] = vb[0];
    }
  }
  if constexpr (LATE) pdl_wait();  // this grid completes after the previous one
}

// ---- Jeff prep: centred per-head RMSNorm + partial RoPE --------------------------------

// CTA per (32-token tile, head). The time-first inputs are read as [head_dim]
// x 32-token runs into shared memory; 32 threads each sum one token's squares
// sequentially (lib.rs:676-683), every element is scaled as
// x * (scale * (1 + w)) (:684-686), the first rotary_dim channels rotated
// (:690-707), and the tile written head-major.
__global__ void __launch_bounds__(256) jeff_prep_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ q_norm, const float* __restrict__ k_norm,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, float* __restrict__ qh,
    float* __restrict__ kh, float* __restrict__ vh, uint32_t length, uint32_t hd,
    uint32_t rotary, float eps) {
  pdl_enter();
  extern __shared__ float tile[];  // [hd][33]
  __shared__ float scale_s[32];
  const uint32_t tid = threadIdx.x, head = blockIdx.y, t0 = blockIdx.x * 32;
  const uint32_t half = rotary / 2;
  const uint64_t feat = uint64_t(head) * hd;
  const float hd_f = float(hd);
  for (int which = 0; which < 3; ++which) {
    const float* src = which == 0 ? q : which == 1 ? k : v;
    float* dst = which == 0 ? qh : which == 1 ? kh : vh;
    for (uint32_t idx = tid; idx < hd * 32; idx += 256) {
      const uint32_t i = idx >> 5, t = idx & 31;
      tile[i * 33 + t] = t0 + t < length ? src[t0 + t + uint64_t(length) * (feat + i)] : 0.0f;
    }
    __syncthreads();
    if (which < 2) {
      const float* w = which == 0 ? q_norm : k_norm;
      if (tid < 32) {
        float ms = 0.0f;
        for (uint32_t i = 0; i < hd; ++i) {
          const float x = tile[i * 33 + tid];
          ms = __fadd_rn(ms, __fmul_rn(x, x));
        }
        ms = __fdiv_rn(ms, hd_f);
        scale_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
      }
      __syncthreads();
      for (uint32_t idx = tid; idx < hd * 32; idx += 256) {
        const uint32_t i = idx >> 5, t = idx & 31;
        tile[i * 33 + t] =
            __fmul_rn(tile[i * 33 + t], __fmul_rn(scale_s[t], __fadd_rn(1.0f, __ldg(w + i))));
      }
      __syncthreads();
      for (uint32_t idx = tid; idx < half * 32; idx += 256) {
        const uint32_t i = idx >> 5, t = idx & 31;
        if (t0 + t < length) {
          const float c = __ldg(cos_t + uint64_t(t0 + t) * half + i);
          const float s = __ldg(sin_t + uint64_t(t0 + t) * half + i);
          const float a = tile[i * 33 + t], b = tile[(i + half) * 33 + t];
          tile[i * 33 + t] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
          tile[(i + half) * 33 + t] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
        }
      }
      __syncthreads();
    }
    for (uint32_t idx = tid; idx < hd * 32; idx += 256) {
      const uint32_t t = idx / hd, i = idx - t * hd;
      if (t0 + t < length) dst[(uint64_t(head) * length + t0 + t) * hd + i] = tile[i * 33 + t];
    }
    __syncthreads();
  }
}

// ---- Jeff attention on the tensor cores ----------------------------------------------
//
// For head_dim a multiple of 32 and a length a multiple of 128, the Jeff block
// runs as tensor-core GEMMs around the masked softmax: S_h = Q_h K_h^T (the
// 3xTF32 GEMM, batched over heads), the causal / active softmax of S, O_h =
// P_h V_h (the same GEMM on V_h transposed), then the gate. Heads holding a
// value that is non-finite or at least 2^40 are redone by the f32 kernel
// (whose arithmetic follows the reference's handling of such values); below
// 2^40 every scaled score is below 2^84, far from the -1e30 the softmax gives
// masked keys and from overflow.

// hi = tf32(x), lo = x - hi (exact, so hi + lo == x); a value beyond the
// largest tf32 (or non-finite) stays whole in hi with lo = 0. bad: |x| >= 2^40
// or non-finite (the head goes to the f32 kernel).
__device__ __forceinline__ void jeff_split(float x, float* hi, float* lo, bool* bad) {
  const bool ok = fabsf(x) < 3.4e38f;
  *bad |= !(fabsf(x) < 1.099511627776e12f);  // 2^40
  *hi = ok ? tf32_round_finite(x) : x;
  *lo = ok ? __fsub_rn(x, *hi) : 0.0f;
}

// The Jeff prep for the tensor-core route, one (32-token, head, tensor) tile
// per CTA (blockIdx.z: 0 q, 1 k, 2 v), with the arithmetic of jeff_prep_kernel
// (bit-identical values). q and k are written as the hi / lo planes of the
// score GEMM's operands, head-major [head][token][HD]; v as the hi / lo planes
// of V^T [head][channel][token] (the P V GEMM's weight; hi + lo == v).
// flags[head] = 1 when a value of the head is non-finite or at least 2^40.
// length % 32 == 0.
template <int HD>
__global__ void __launch_bounds__(256) jeff_prep_planes_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ q_norm, const float* __restrict__ k_norm,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, float* __restrict__ qhi,
    float* __restrict__ qlo, float* __restrict__ khi, float* __restrict__ klo,
    float* __restrict__ vthi, float* __restrict__ vtlo, uint32_t length, uint32_t rotary, float eps,
    uint8_t* flags) {
  pdl_enter();
  __shared__ float tile[HD * 33];
  __shared__ float scale_s[32];
  const uint32_t tid = threadIdx.x, head = blockIdx.y, t0 = blockIdx.x * 32, which = blockIdx.z;
  const uint64_t feat = uint64_t(head) * HD;
  const float* src = which == 0 ? q : which == 1 ? k : v;
  bool bad = false;
  // eight loads in flight per thread before their shared-memory stores
#pragma unroll
  for (uint32_t idx0 = tid; idx0 < HD * 32; idx0 += 256 * 8) {
    float r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t idx = idx0 + 256 * u, i = idx >> 5, t = idx & 31;
      r[u] = src[t0 + t + uint64_t(length) * (feat + i)];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const uint32_t idx = idx0 + 256 * u;
      tile[(idx >> 5) * 33 + (idx & 31)] = r[u];
    }
  }
  __syncthreads();
  if (which == 2) {
    // V^T planes: row (head, channel i), 32 consecutive tokens per warp
#pragma unroll 4
    for (uint32_t idx = tid; idx < HD * 32; idx += 256) {
      const uint32_t i = idx >> 5, t = idx & 31;
      float h, l;
      jeff_split(tile[i * 33 + t], &h, &l, &bad);
      const uint64_t o = (feat + i) * length + t0 + t;
      vthi[o] = h;
      vtlo[o] = l;
    }
  } else {
    const float* w = which == 0 ? q_norm : k_norm;
    if (tid < 32) {
      float ms = 0.0f;
#pragma unroll 16
      for (uint32_t i = 0; i < HD; ++i) {
        const float x = tile[i * 33 + tid];
        ms = __fadd_rn(ms, __fmul_rn(x, x));
      }
      ms = __fdiv_rn(ms, float(HD));
      scale_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
    }
    __syncthreads();
#pragma unroll 4
    for (uint32_t idx = tid; idx < HD * 32; idx += 256) {
      const uint32_t i = idx >> 5, t = idx & 31;
      tile[i * 33 + t] =
          __fmul_rn(tile[i * 33 + t], __fmul_rn(scale_s[t], __fadd_rn(1.0f, __ldg(w + i))));
    }
    __syncthreads();
    const uint32_t half = rotary / 2;
    for (uint32_t idx = tid; idx < half * 32; idx += 256) {
      const uint32_t i = idx >> 5, t = idx & 31;
      const float c = __ldg(cos_t + uint64_t(t0 + t) * half + i);
      const float sn = __ldg(sin_t + uint64_t(t0 + t) * half + i);
      const float a = tile[i * 33 + t], b = tile[(i + half) * 33 + t];
      tile[i * 33 + t] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
      tile[(i + half) * 33 + t] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
    }
    __syncthreads();
    float* dhi = which == 0 ? qhi : khi;
    float* dlo = which == 0 ? qlo : klo;
#pragma unroll 4
    for (uint32_t idx = tid; idx < HD * 32; idx += 256) {
      const uint32_t t = idx / HD, i = idx % HD;
      float h, l;
      jeff_split(tile[i * 33 + t], &h, &l, &bad);
      const uint64_t o = (uint64_t(head) * length + t0 + t) * HD + i;
      dhi[o] = h;
      dlo[o] = l;
    }
  }
  if (__syncthreads_or(bad) && tid == 0) flags[head] = 1;
}

// keep[k] = (active[k] != 0); *first = the smallest such k (untouched when
// none): query q has a kept key (causal) exactly when q >= *first.
__global__ void __launch_bounds__(256) jeff_keep_kernel(const float* __restrict__ active,
                                                        uint8_t* __restrict__ keep, int* first,
                                                        uint32_t length) {
  pdl_enter();
  for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < length;
       k += gridDim.x * blockDim.x) {
    const bool on = active[k] != 0.0f;
    keep[k] = on;
    if (on) atomicMin(first, int(k));
  }
}

// exp(d) for d <= 0 as 2^(d log2 e) on the ex2 unit (relative error ~2^-22
// plus |d| 2^-24 from the product; results below 2^-126 flush to 0).
__device__ __forceinline__ float jeff_exp(float d) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fmul_rn(d, 1.4426950408889634f)));
  return r;
}

// The causal / active softmax of one score row per warp, written as the
// hi / lo planes of the P V GEMM's x operand. Row = (head, query q) of
// scores [head][q][key] (keys contiguous, only keys <= q read); keys [0, W),
// W = rt (q / rt + 1), are written (the P V contraction of q's rt-query tile
// row stops there; rt = 128, or 256 when that GEMM runs on CTA pairs): p = exp(s scale - max) / sum over the kept keys (key <=
// q and keep[key]), 0 for the others. Two passes over the row: a running
// (max, sum) per lane, combined over the warp, then the probabilities (the
// second read comes from cache). Rows q < *first have no kept key and are
// written as zeros (their output is 0).
__global__ void __launch_bounds__(256) jeff_softmax_planes_kernel(
    const float* __restrict__ scores, const uint8_t* __restrict__ keep, const int* first,
    float* __restrict__ phi, float* __restrict__ plo, uint32_t length, uint32_t rows, float scale,
    uint32_t rt) {
  pdl_enter();
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint32_t qi = row % length;
  const uint32_t width = (qi / rt + 1) * rt;
  const float* srow = scores + uint64_t(row) * length;
  float* hrow = phi + uint64_t(row) * length;
  float* lrow = plo + uint64_t(row) * length;
  if (int(qi) < __ldg(first)) {
    const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (uint32_t c = 4 * lane; c < width; c += 128) {
      *reinterpret_cast<float4*>(hrow + c) = z;
      *reinterpret_cast<float4*>(lrow + c) = z;
    }
    return;
  }
  // the scaled scores of keys c .. c + 3, -inf when not kept
  auto scaled = [&](uint32_t c, float* v) {
    const float4 sv = __ldg(reinterpret_cast<const float4*>(srow + c));
    const uint32_t kb = __ldg(reinterpret_cast<const uint32_t*>(keep + c));
    const float x[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool kept = c + j <= qi && ((kb >> (8 * j)) & 0xFFu) != 0;
      v[j] = kept ? __fmul_rn(x[j], scale) : -INFINITY;
    }
  };
  float mx = -INFINITY, sum = 0.0f;
#pragma unroll 8
  for (uint32_t c = 4 * lane; c <= qi; c += 128) {
    float v[4];
    scaled(c, v);
    const float m4 = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
    if (m4 > mx) {  // a new running max: rescale the lane's sum
      sum = mx == -INFINITY ? 0.0f : __fmul_rn(sum, jeff_exp(__fsub_rn(mx, m4)));
      mx = m4;
    }
    if (mx != -INFINITY) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (v[j] != -INFINITY) sum = __fadd_rn(sum, jeff_exp(__fsub_rn(v[j], mx)));
    }
  }
  const float m = warp_max(mx);  // finite: key *first <= q is kept
  sum = mx == -INFINITY ? 0.0f : __fmul_rn(sum, jeff_exp(__fsub_rn(mx, m)));
  sum = warp_sum(sum);
  const float r = __fdiv_rn(1.0f, sum);
#pragma unroll 4
  for (uint32_t c = 4 * lane; c < width; c += 128) {
    float h[4] = {0.0f, 0.0f, 0.0f, 0.0f}, l[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (c <= qi) {
      float v[4];
      scaled(c, v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float pv = v[j] == -INFINITY ? 0.0f : __fmul_rn(jeff_exp(__fsub_rn(v[j], m)), r);
        h[j] = tf32_round_finite(pv);
        l[j] = __fsub_rn(pv, h[j]);
      }
    }
    *reinterpret_cast<float4*>(hrow + c) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lrow + c) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// The Jeff output, elementwise over out (hidden, length): the sum of the P V
// GEMM's slots for this element (slot p at o + p * n, p < split.pieces(head,
// t / split.row_tokens), added in slot order), 0 for tokens t < *first (no kept key), then
// times sigmoid(gate). One warp per 128 tokens of a feature row (one query
// tile: one piece count per warp), four consecutive tokens per lane.
__global__ void __launch_bounds__(256) jeff_gate_kernel(const float* __restrict__ o,
                                                        const float* __restrict__ gate,
                                                        float* __restrict__ out, const int* first,
                                                        uint64_t n, uint32_t length, uint32_t hd,
                                                        uint32_t nwarps, CausalKSplit split) {
  pdl_enter();
  const int kfirst = __ldg(first);
  const uint32_t lane = threadIdx.x & 31, tiles = length / 128;
  for (uint32_t w = blockIdx.x * 8 + (threadIdx.x >> 5); w < nwarps; w += gridDim.x * 8) {
    const uint32_t f = w / tiles, lm = w - f * tiles;
    uint32_t pieces = 0;
    if (lane == 0) pieces = split.pieces(f / hd, lm * 128 / split.row_tokens);
    pieces = __shfl_sync(0xffffffffu, pieces, 0);
    const uint32_t t = lm * 128 + lane * 4;
    const uint64_t i = uint64_t(f) * length + t;
    float4 v = __ldg(reinterpret_cast<const float4*>(o + i));
    for (uint32_t p = 1; p < pieces; ++p) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(o + i + p * n));
      v = make_float4(__fadd_rn(v.x, u.x), __fadd_rn(v.y, u.y), __fadd_rn(v.z, u.z),
                      __fadd_rn(v.w, u.w));
    }
    const float4 g = ld_stream(reinterpret_cast<const float4*>(gate + i));
    const float x[4] = {v.x, v.y, v.z, v.w}, gg[4] = {g.x, g.y, g.z, g.w};
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      y[j] = int(t) + j < kfirst
                 ? 0.0f
                 : __fmul_rn(x[j], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gg[j]))));
    *reinterpret_cast<float4*>(out + i) = make_float4(y[0], y[1], y[2], y[3]);
  }
}

// ---- attention -----------------------------------------------------------------------

struct AttnArgs {
  const float* q;
  const float* k;
  const float* v;
  float* out;
  const uint8_t* keep;
  const float* bias;
  const float* active;
  const float* gate;
  int64_t gate_offset, out_tok, out_feat, out_batch;
  uint32_t heads, length, hd;
  float scale;
  int empty_nan, causal;
  int64_t window, valid_len;
  // (batch*heads) flags: V of that head holds a non-finite value. The tensor
  // core kernel leaves those heads (vflag_mode 1) to the f32 kernel, which
  // then runs on them only (vflag_mode 2); 0 = no routing.
  const uint8_t* vflags;
  int vflag_mode;
  // head_dim 64 only: q, k, v as tile images (nqt / nkt tiles per head)
  // instead of the head-major q / k / v, when qimg is set
  const uint8_t* qimg = nullptr;
  const uint8_t* kimg = nullptr;
  const uint8_t* vimg = nullptr;
  uint32_t nqt = 0, nkt = 0;
  // the mask digest, when computed before the call (attn_keep_digest_kernel)
  const uint32_t* digest_words = nullptr;
  const uint8_t* digest_summary = nullptr;
  // q = q + q_lo and k = k + k_lo when set (hi / lo planes, same layout)
  const float* q_lo = nullptr;
  const float* k_lo = nullptr;
  // when set, v and v_lo are the hi / lo planes of V^T: channel c of key j of
  // head bh at (bh * hd + c) * length + j
  const float* v_lo = nullptr;
};

// Channels ch .. ch + 3 of row `row` of head bh of q (t = 0), k (1) or v (2):
// from the head-major tensor, or hi + lo of its tile image (exact: the image
// keeps hi + lo == x for every value).
__device__ __forceinline__ float4 attn_ld4(const AttnArgs& a, int t, uint64_t bh, uint32_t row,
                                           uint32_t ch) {
  if (a.qimg) {
    const uint8_t* tile;
    uint32_t plane, off;
    if (t == 0) {
      tile = a.qimg + (bh * a.nqt + row / kWsTQ) * (2 * kWsQPlane);
      plane = kWsQPlane;
      off = img_kmajor_off(row % kWsTQ, ch, kWsQRegion);
    } else {
      tile = (t == 1 ? a.kimg : a.vimg) + (bh * a.nkt + row / kWsKB) * kWsSlot;
      plane = kWsTile;
      off = t == 1 ? img_kmajor_off(row % kWsKB, ch, kWsKRegion) : img_v_off(row % kWsKB, ch);
    }
    const float4 h = __ldg(reinterpret_cast<const float4*>(tile + off));
    const float4 l = __ldg(reinterpret_cast<const float4*>(tile + plane + off));
    return make_float4(__fadd_rn(h.x, l.x), __fadd_rn(h.y, l.y), __fadd_rn(h.z, l.z),
                       __fadd_rn(h.w, l.w));
  }
  const float* src = t == 0 ? a.q : t == 1 ? a.k : a.v;
  if (t == 2 && a.v_lo) {  // V^T planes: four channels, length apart
    const uint64_t o = (bh * a.hd + ch) * a.length + row;
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      x[i] = __fadd_rn(__ldg(a.v + o + uint64_t(i) * a.length),
                       __ldg(a.v_lo + o + uint64_t(i) * a.length));
    return make_float4(x[0], x[1], x[2], x[3]);
  }
  const uint64_t off = (bh * a.length + row) * a.hd + ch;
  const float* lo = t == 0 ? a.q_lo : t == 1 ? a.k_lo : nullptr;
  const float4 h = ld_stream(reinterpret_cast<const float4*>(src + off));
  if (!lo) return h;
  const float4 l = ld_stream(reinterpret_cast<const float4*>(lo + off));
  return make_float4(__fadd_rn(h.x, l.x), __fadd_rn(h.y, l.y), __fadd_rn(h.z, l.z),
                     __fadd_rn(h.w, l.w));
}

__device__ __forceinline__ bool routed_away(const AttnArgs& a, uint32_t bh) {
  if (a.vflag_mode == 1) return a.vflags[bh] != 0;
  if (a.vflag_mode == 2) return a.vflags[bh] == 0;
  return false;
}

// Keys [lo, hi) that the analytic conditions allow for queries [q0, q1].
__device__ __forceinline__ void analytic_range(const AttnArgs& a, int64_t q0, int64_t q1,
                                               int64_t* lo, int64_t* hi) {
  int64_t l = 0, h = a.length;
  if (a.causal) h = min(h, q1 + 1);
  if (a.window >= 0) {
    l = max(l, q0 - a.window);
    h = min(h, q1 + a.window + 1);
  }
  if (a.valid_len >= 0) h = min(h, a.valid_len);
  *lo = l;
  *hi = max(l, h);
}

__device__ __forceinline__ bool key_kept(const AttnArgs& a, uint32_t b, int64_t qi, int64_t kj) {
  if (a.causal && kj > qi) return false;
  if (a.window >= 0 && (kj < qi - a.window || kj > qi + a.window)) return false;
  if (a.valid_len >= 0 && kj >= a.valid_len) return false;
  const uint64_t L = a.length;
  if (a.keep && a.keep[uint64_t(qi) + L * (uint64_t(kj) + L * b)] == 0) return false;
  if (a.active && a.active[uint64_t(b) * L + kj] == 0.0f) return false;
  return true;
}

// out element for (token qi, feature f, batch b); empty / +inf rows take
// the empty value; the gate multiplies every written value.
__device__ __forceinline__ void store_out(const AttnArgs& a, uint32_t b, uint32_t qi,
                                          uint64_t f, float val) {
  const int64_t idx = int64_t(qi) * a.out_tok + int64_t(f) * a.out_feat + int64_t(b) * a.out_batch;
  if (a.gate) {
    const float g = a.gate[a.gate_offset + idx];
    val = __fmul_rn(val, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
  }
  a.out[idx] = val;
}

// Narrows [lo, hi) to the keys the keep mask allows for some query of
// [q0, q0 + nq); every thread of the CTA gets the result.
__device__ void keep_narrow(const AttnArgs& a, uint32_t b, uint32_t q0, uint32_t nq, int64_t* lo,
                            int64_t* hi, int* red) {
  if (threadIdx.x == 0) {
    red[0] = int(*hi);
    red[1] = int(*lo) - 1;
  }
  __syncthreads();
  const uint64_t L = a.length;
  for (int64_t kj = *lo + threadIdx.x; kj < *hi; kj += blockDim.x) {
    const uint8_t* row = a.keep + uint64_t(q0) + L * (uint64_t(kj) + L * b);
    bool any = false;
    for (uint32_t i = 0; i < nq && !any; ++i) any = row[i] != 0;
    if (any) {
      atomicMin(&red[0], int(kj));
      atomicMax(&red[1], int(kj));
    }
  }
  __syncthreads();
  const int first = red[0], last = red[1];
  __syncthreads();
  if (first > last) {
    *hi = *lo;
  } else {
    *lo = first;
    *hi = int64_t(last) + 1;
  }
}

constexpr int kQT = 64;  // queries per CTA

// Flash kernel: 256 threads as 16 x 16; thread (ty, tx) owns queries
// 4ty..4ty+3, keys KT*tx.. of each block and output channels
// 64*j + 4tx..4tx+3. Shared memory: Q^T [HD][64], K^T [HD][KB], V [KB][HD],
// P [64][KB + 4].
template <int HD, int KB>
__global__ void __launch_bounds__(256) attn_flash_kernel(AttnArgs a) {
  constexpr int KT = KB / 16;
  constexpr int DJ = HD / 64;
  constexpr int PS = KB + 4;
  extern __shared__ __align__(16) float sm[];
  float* Qt = sm;
  float* Kt = Qt + HD * kQT;
  float* Vs = Kt + HD * KB;
  float* Ps = Vs + KB * HD;
  __shared__ int red[2];
  __shared__ int vbad;
  pdl_enter();
  const uint32_t tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const uint32_t head = blockIdx.y, b = blockIdx.z;
  if (routed_away(a, b * a.heads + head)) return;
  // query tiles q0 = 64 blockIdx.x, then gridDim.x tiles further on (a grid
  // of one tile per head runs them all)
  for (uint32_t q0 = blockIdx.x * kQT; q0 < a.length; q0 += gridDim.x * kQT) {
    const uint32_t L = a.length;
    const uint32_t nq = min(uint32_t(kQT), L - q0);
    const uint64_t bh = uint64_t(b) * a.heads + head;
    int64_t lo, hi;
    analytic_range(a, q0, q0 + nq - 1, &lo, &hi);
    if (a.keep && lo < hi) keep_narrow(a, b, q0, nq, &lo, &hi, red);

    for (uint32_t idx = tid; idx < kQT * HD / 4; idx += 256) {
      const uint32_t qq = idx % kQT, h4 = idx / kQT;
      float4 val = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (qq < nq) val = attn_ld4(a, 0, bh, q0 + qq, 4 * h4);
      Qt[(4 * h4 + 0) * kQT + qq] = val.x;
      Qt[(4 * h4 + 1) * kQT + qq] = val.y;
      Qt[(4 * h4 + 2) * kQT + qq] = val.z;
      Qt[(4 * h4 + 3) * kQT + qq] = val.w;
    }

    float o[4][DJ][4];
    float m[4], l[4];
    bool inf_row[4];
  #pragma unroll
    for (int i = 0; i < 4; ++i) {
      m[i] = -INFINITY;
      l[i] = 0.0f;
      inf_row[i] = false;
  #pragma unroll
      for (int j = 0; j < DJ; ++j)
  #pragma unroll
        for (int e = 0; e < 4; ++e) o[i][j][e] = 0.0f;
    }

    const int64_t kb_first = lo / KB * KB;
    for (int64_t kb0 = kb_first; kb0 < hi; kb0 += KB) {
      if (tid == 0) vbad = 0;
      __syncthreads();  // the previous block's reads of K, V, P are done
      for (uint32_t idx = tid; idx < KB * HD / 4; idx += 256) {
        const uint32_t kk = idx % KB, h4 = idx / KB;
        float4 val = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (kb0 + kk < L)
          val = attn_ld4(a, 1, bh, uint32_t(kb0 + kk), 4 * h4);
        Kt[(4 * h4 + 0) * KB + kk] = val.x;
        Kt[(4 * h4 + 1) * KB + kk] = val.y;
        Kt[(4 * h4 + 2) * KB + kk] = val.z;
        Kt[(4 * h4 + 3) * KB + kk] = val.w;
      }
      bool bad = false;
      for (uint32_t idx = tid; idx < KB * HD / 4; idx += 256) {
        const uint32_t kk = idx / (HD / 4), h4 = idx % (HD / 4);
        float4 val = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (kb0 + kk < L)
          val = attn_ld4(a, 2, bh, uint32_t(kb0 + kk), 4 * h4);
        bad |= !(fabsf(val.x) < INFINITY && fabsf(val.y) < INFINITY && fabsf(val.z) < INFINITY &&
                 fabsf(val.w) < INFINITY);
        *reinterpret_cast<float4*>(Vs + kk * HD + 4 * h4) = val;
      }
      if (bad) vbad = 1;
      __syncthreads();

      // scores of queries 4ty+i against keys KT*tx+j
      float s[4][KT];
  #pragma unroll
      for (int i = 0; i < 4; ++i)
  #pragma unroll
        for (int j = 0; j < KT; ++j) s[i][j] = 0.0f;
  #pragma unroll 8
      for (int h = 0; h < HD; ++h) {
        const float4 q4 = *reinterpret_cast<const float4*>(Qt + h * kQT + 4 * ty);
        float kv[KT];
        if constexpr (KT == 4) {
          const float4 k4 = *reinterpret_cast<const float4*>(Kt + h * KB + 4 * tx);
          kv[0] = k4.x; kv[1] = k4.y; kv[2] = k4.z; kv[3] = k4.w;
        } else {
          const float2 k2 = *reinterpret_cast<const float2*>(Kt + h * KB + 2 * tx);
          kv[0] = k2.x; kv[1] = k2.y;
        }
        const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
  #pragma unroll
        for (int i = 0; i < 4; ++i)
  #pragma unroll
          for (int j = 0; j < KT; ++j) s[i][j] = __fmaf_rn(qv[i], kv[j], s[i][j]);
      }

      // mask, scale, online softmax
  #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t qi = int64_t(q0) + 4 * ty + i;
        float mb = -INFINITY;
  #pragma unroll
        for (int j = 0; j < KT; ++j) {
          const int64_t kj = kb0 + KT * tx + j;
          float sc = -INFINITY;
          if (qi < L && kj >= lo && kj < hi && key_kept(a, b, qi, kj)) {
            sc = __fmul_rn(s[i][j], a.scale);
            if (a.bias) sc = __fadd_rn(sc, a.bias[uint64_t(qi) + uint64_t(L) * (uint64_t(kj) + uint64_t(L) * b)]);
            if (sc == INFINITY) inf_row[i] = true;
            if (!(fabsf(sc) < INFINITY)) sc = -INFINITY;  // NaN / inf: contributes nothing
          }
          s[i][j] = sc;
          mb = fmaxf(mb, sc);
        }
  #pragma unroll
        for (int d = 1; d < 16; d <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, d));
        const float mn = fmaxf(m[i], mb);
        float corr = 1.0f, ps = 0.0f;
        if (mn != -INFINITY) {
          corr = expf(__fsub_rn(m[i], mn));
  #pragma unroll
          for (int j = 0; j < KT; ++j) {
            const float p = s[i][j] == -INFINITY ? 0.0f : expf(__fsub_rn(s[i][j], mn));
            s[i][j] = p;
            ps = __fadd_rn(ps, p);
          }
        } else {
  #pragma unroll
          for (int j = 0; j < KT; ++j) s[i][j] = 0.0f;
        }
  #pragma unroll
        for (int d = 1; d < 16; d <<= 1) ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, d));
        m[i] = mn;
        l[i] = __fmaf_rn(l[i], corr, ps);
  #pragma unroll
        for (int j = 0; j < DJ; ++j)
  #pragma unroll
          for (int e = 0; e < 4; ++e) o[i][j][e] = __fmul_rn(o[i][j][e], corr);
        if constexpr (KT == 4) {
          *reinterpret_cast<float4*>(Ps + (4 * ty + i) * PS + 4 * tx) =
              make_float4(s[i][0], s[i][1], s[i][2], s[i][3]);
        } else {
          *reinterpret_cast<float2*>(Ps + (4 * ty + i) * PS + 2 * tx) = make_float2(s[i][0], s[i][1]);
        }
      }
      __syncthreads();

      // O += P V (keys whose p is 0 are skipped when V holds a non-finite value)
      const bool guard = vbad != 0;
  #pragma unroll 2
      for (int k4 = 0; k4 < KB; k4 += 4) {
        float p[4][4];
  #pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 t = *reinterpret_cast<const float4*>(Ps + (4 * ty + i) * PS + k4);
          p[i][0] = t.x; p[i][1] = t.y; p[i][2] = t.z; p[i][3] = t.w;
        }
  #pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
  #pragma unroll
          for (int j = 0; j < DJ; ++j) {
            const float4 vv = *reinterpret_cast<const float4*>(Vs + (k4 + kk) * HD + 64 * j + 4 * tx);
            const float ve[4] = {vv.x, vv.y, vv.z, vv.w};
  #pragma unroll
            for (int i = 0; i < 4; ++i) {
              if (guard && p[i][kk] == 0.0f) continue;
  #pragma unroll
              for (int e = 0; e < 4; ++e) o[i][j][e] = __fmaf_rn(p[i][kk], ve[e], o[i][j][e]);
            }
          }
        }
      }
    }

    // a +inf score seen by any of the 16 lanes of a row empties the whole row
  #pragma unroll
    for (int i = 0; i < 4; ++i)
  #pragma unroll
      for (int d = 1; d < 16; d <<= 1)
        inf_row[i] = (__shfl_xor_sync(0xffffffffu, int(inf_row[i]), d) != 0) || inf_row[i];
  #pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t qi = q0 + 4 * ty + i;
      if (qi >= L) continue;
      const bool empty = l[i] == 0.0f || inf_row[i];
      const float ev = a.empty_nan ? NAN : 0.0f;
  #pragma unroll
      for (int j = 0; j < DJ; ++j)
  #pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t d = 64 * j + 4 * tx + e;
          const float val = empty ? ev : __fdiv_rn(o[i][j][e], l[i]);
          store_out(a, b, qi, uint64_t(head) * HD + d, val);
        }
    }
    __syncthreads();  // the shared tiles are reused by the next query tile
  }
}

// Any head_dim: CTA per (query, head, batch), scores of the whole row in
// shared memory (length floats), the reference's fused_attention structure.
__global__ void __launch_bounds__(128) attn_row_kernel(AttnArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* scores = sm;                // [length]
  float* query = sm + a.length;      // [hd]
  __shared__ float scratch[4];
  __shared__ int inf_flag;
  pdl_enter();
  const uint32_t qi = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  if (routed_away(a, b * a.heads + head)) return;
  const uint32_t L = a.length, hd = a.hd;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t base = (uint64_t(b) * a.heads + head) * L * hd;
  if (threadIdx.x == 0) inf_flag = 0;
  for (uint32_t d = threadIdx.x; d < hd; d += 128) query[d] = a.q[base + uint64_t(qi) * hd + d];
  __syncthreads();
  int64_t lo, hi;
  analytic_range(a, qi, qi, &lo, &hi);
  for (uint32_t kj = warp; kj < L; kj += 4) {
    const bool kept = kj >= lo && kj < hi && key_kept(a, b, qi, kj);
    float dot = 0.0f;
    if (kept) {
      const float* kr = a.k + base + uint64_t(kj) * hd;
      for (uint32_t d = lane; d < hd; d += 32) dot = __fmaf_rn(query[d], kr[d], dot);
      dot = warp_sum(dot);
    }
    if (lane == 0) {
      float sc = -INFINITY;
      if (kept) {
        sc = __fmul_rn(dot, a.scale);
        if (a.bias) sc = __fadd_rn(sc, a.bias[uint64_t(qi) + uint64_t(L) * (uint64_t(kj) + uint64_t(L) * b)]);
        if (sc == INFINITY) inf_flag = 1;
        if (!(fabsf(sc) < INFINITY)) sc = -INFINITY;
      }
      scores[kj] = sc;
    }
  }
  __syncthreads();
  float mx = -INFINITY;
  for (uint32_t kj = threadIdx.x; kj < L; kj += 128) mx = fmaxf(mx, scores[kj]);
  mx = warp_max(mx);
  if (lane == 0) scratch[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(scratch[0], scratch[1]), fmaxf(scratch[2], scratch[3]));
  __syncthreads();
  float sum = 0.0f;
  for (uint32_t kj = threadIdx.x; kj < L; kj += 128) {
    const float sc = scores[kj];
    const float p = sc == -INFINITY ? 0.0f : expf(__fsub_rn(sc, mx));
    scores[kj] = p;
    sum = __fadd_rn(sum, p);
  }
  sum = warp_sum(sum);
  if (lane == 0) scratch[warp] = sum;
  __syncthreads();
  sum = __fadd_rn(__fadd_rn(scratch[0], scratch[1]), __fadd_rn(scratch[2], scratch[3]));
  const bool empty = sum == 0.0f || inf_flag;
  for (uint32_t d = threadIdx.x; d < hd; d += 128) {
    float acc = 0.0f;
    if (!empty) {
      const float* vc = a.v + base + d;
      for (uint32_t kj = 0; kj < L; ++kj) {
        const float p = scores[kj];
        if (p != 0.0f) acc = __fmaf_rn(p, vc[uint64_t(kj) * hd], acc);
      }
    }
    const float val = empty ? (a.empty_nan ? NAN : 0.0f) : __fdiv_rn(acc, sum);
    store_out(a, b, qi, uint64_t(head) * hd + d, val);
  }
}


// ---- tensor-core attention (head_dim 64) ---------------------------------------------

constexpr int kTQ = 128;                  // queries per CTA of the tensor-core kernel
constexpr long long kTcWait = 1LL << 31;  // bound of every wait (SM cycles)

__device__ uint32_t g_tc_wait_timeouts;

#include "attn_ws.cuh"
static_assert(kWsTQ == kTQ, "the grid tiles the queries by 128");

// The tensor-core path for head_dim 64: attn_img_split_kernel writes the tile
// images (and, when pre_flags is null, the per-head flags of values the
// tensor cores cannot take), attn_ws_kernel computes every unflagged head,
// attn_flash_kernel the flagged ones. pre_flags: flags already computed on the
// stream (the Laya prep kernel sets them). When a.qimg is set, the images
// exist already (the Laya prep kernel wrote them, with pre_flags) and q, k,
// v are not read. Returns 1 when the shape is not covered (nothing launched).
// TFX_ATTN_KERNEL=f32: the f32-pipe kernel for every head (read once).
bool attn_f32_only() {
  static const bool f32_only = [] {
    const char* e = getenv("TFX_ATTN_KERNEL");
    return e && std::string(e) == "f32";
  }();
  return f32_only;
}

bool attn_tc_covers(uint32_t hd, uint64_t rows, const DeviceInfo& dev) {
  return !attn_f32_only() && hd == 64 && rows < (uint64_t(1) << 31) && kWsSmem <= size_t(dev.smem_optin);
}

int attn_launch_tc(const char* op, AttnArgs a, uint32_t batch, const DeviceInfo& dev,
                   cudaStream_t stream, const uint8_t* pre_flags) {
  const uint64_t rows = uint64_t(batch) * a.heads * a.length;
  const bool have_img = a.qimg != nullptr;
  if (!attn_tc_covers(a.hd, rows, dev) ||
      (!have_img && (!aligned(a.q, 16) || !aligned(a.k, 16) || !aligned(a.v, 16))))
    return 1;
  const uint32_t nbh = batch * a.heads;
  // scratch: the flags (unless given), then the tile images of q, k, v (hi
  // and lo, padded to whole tiles: 512 bytes per padded row and tensor)
  const uint32_t lq = (a.length + kWsTQ - 1) / kWsTQ * kWsTQ;
  const uint32_t lk = (a.length + kWsKB - 1) / kWsKB * kWsKB;
  const size_t qimg_bytes = have_img ? 0 : size_t(nbh) * lq * 512;
  const size_t kimg_bytes = have_img ? 0 : size_t(nbh) * lk * 512;
  const size_t flag_bytes = pre_flags ? 0 : (size_t(nbh) + 255) / 256 * 256;
  // the mask digest (keep / active): 1 KB of words and one summary byte per
  // (batch, query tile, key tile)
  const bool mask = a.keep || a.active;
  const bool have_digest = a.digest_words != nullptr;
  const uint32_t nqt = lq / kWsTQ, nkt = lk / kWsKB;
  const size_t digest_tiles = mask && !have_digest ? size_t(batch) * nqt * nkt : 0;
  const size_t words_bytes = digest_tiles * 1024;
  const size_t summary_bytes = (digest_tiles + 255) / 256 * 256;
  uint8_t* scratch = nullptr;
  cudaError_t e = scratch_malloc(reinterpret_cast<void**>(&scratch),
                                 flag_bytes + qimg_bytes + 2 * kimg_bytes + words_bytes +
                                     summary_bytes,
                                 stream);
  if (e == cudaSuccess && flag_bytes) e = cudaMemsetAsync(scratch, 0, nbh, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  }
  uint8_t* flags = pre_flags ? nullptr : scratch;
  uint8_t* own = scratch + flag_bytes;
  const uint8_t* qimg = have_img ? a.qimg : own;
  const uint8_t* kimg = have_img ? a.kimg : own + qimg_bytes;
  const uint8_t* vimg = have_img ? a.vimg : own + qimg_bytes + kimg_bytes;
  uint32_t* own_words = reinterpret_cast<uint32_t*>(own + qimg_bytes + 2 * kimg_bytes);
  uint8_t* own_summary = reinterpret_cast<uint8_t*>(own_words) + words_bytes;
  const uint32_t* words = have_digest ? a.digest_words : own_words;
  const uint8_t* summary = have_digest ? a.digest_summary : own_summary;
  int rc = TFX_OK;
  if (!have_img) {
    const uint64_t total = uint64_t(nbh) * lq * 16;
    const unsigned blocks =
        unsigned(std::min<uint64_t>((total + 255) / 256, uint64_t(dev.sms) * 16));
    rc = launch_kernel(op, attn_img_split_kernel, dim3(blocks), dim3(256), 0, stream, 1, a.q, a.k,
                       a.v, own, own + qimg_bytes, own + qimg_bytes + kimg_bytes, a.length, lq,
                       lk, total, flags);
  }
  if (rc == TFX_OK && mask && !have_digest)
    rc = launch_kernel(op, attn_keep_digest_kernel, dim3(nkt, nqt, batch), dim3(32), 0, stream, 1,
                       a, nqt, nkt, own_words, own_summary);
  if (rc == TFX_OK) {
    a.vflags = pre_flags ? pre_flags : flags;
    a.vflag_mode = 1;
    const dim3 grid(nqt, a.heads, batch);
    auto run = [&](auto kernel) -> int {
      const cudaError_t e2 = cudaFuncSetAttribute(
          kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kWsSmem));
      if (e2 != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(e2));
      return launch_kernel(op, kernel, grid, dim3(kWsThreads), kWsSmem, stream, 1, qimg, kimg,
                           vimg, nkt, words, summary, a);
    };
    switch ((mask ? 2 : 0) | (a.bias ? 1 : 0)) {
      case 0: rc = run(attn_ws_kernel<false, false>); break;
      case 1: rc = run(attn_ws_kernel<false, true>); break;
      case 2: rc = run(attn_ws_kernel<true, false>); break;
      default: rc = run(attn_ws_kernel<true, true>); break;
    }
  }
  if (rc == TFX_OK) {
    // heads holding a value the tensor cores cannot take: the f32 kernel,
    // which skips the keys whose probability is 0 (the reference's rule)
    a.vflag_mode = 2;
    const size_t fsmem = size_t(64 * 64 * 3 + 64 * 68) * 4;
    const cudaError_t fe = cudaFuncSetAttribute(
        attn_flash_kernel<64, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(fsmem));
    // one CTA per head, looping over the query tiles: the usual call has no
    // flagged head, and a small grid that returns at once costs least
    rc = fe != cudaSuccess ? fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(fe))
                           : launch_kernel(op, attn_flash_kernel<64, 64>, dim3(1, a.heads, batch),
                                           dim3(256), fsmem, stream, 1, a);
  }
  cudaFreeAsync(scratch, stream);
  return rc;
}

// f32_only: skip the tensor-core kernel (a redo of flagged heads).
int attn_launch(const char* op, const AttnArgs& a, uint32_t batch, cudaStream_t stream,
                const uint8_t* pre_flags, bool f32_only = false) {
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  if (!f32_only) {
    const int rc = attn_launch_tc(op, a, batch, dev, stream, pre_flags);
    if (rc != 1) return rc;
  }
  const bool vec = aligned(a.q, 16) && aligned(a.k, 16) && aligned(a.v, 16);
  // a redo of flagged heads: one CTA per head looping over the query tiles
  const dim3 grid(f32_only ? 1u : (a.length + kQT - 1) / kQT, a.heads, batch);
  auto flash = [&](auto kernel, int hd, int kb) -> int {
    const size_t smem = size_t(hd * kQT + hd * kb + kb * hd + kQT * (kb + 4)) * 4;
    if (smem > size_t(dev.smem_optin)) return 1;
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(e));
    return launch_kernel(op, kernel, grid, dim3(256), smem, stream, 1, a);
  };
  if (vec && a.hd == 64) return flash(attn_flash_kernel<64, 64>, 64, 64);
  if (vec && a.hd == 128) return flash(attn_flash_kernel<128, 64>, 128, 64);
  if (vec && a.hd == 256) {
    const int rc = flash(attn_flash_kernel<256, 32>, 256, 32);
    if (rc != 1) return rc;
  }
  const size_t smem = size_t(a.length + a.hd) * 4;
  if (smem > size_t(dev.smem_optin))
    return fail(TFX_ERR_UNSUPPORTED, op, "length",
                "rows longer than the shared-memory score buffer for head_dim " +
                    std::to_string(a.hd));
  const cudaError_t e = cudaFuncSetAttribute(
      attn_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(e));
  return launch_kernel(op, attn_row_kernel, dim3(a.length, a.heads, batch), dim3(128), smem,
                       stream, 1, a);
}

}  // namespace

// ---- host entry points ---------------------------------------------------------------

// Bounded waits of the tensor-core attention that gave up on the current device.
int attention_wait_timeouts(uint32_t* count) {
  const cudaError_t err = cudaMemcpyFromSymbol(count, g_tc_wait_timeouts, sizeof(uint32_t));
  return err == cudaSuccess ? TFX_OK : fail(TFX_ERR_CUDA, "tfx", "wait timeouts", cudaGetErrorString(err));
}

// img (optional): the tensor-core attention's tile images (q, k, v) to write
// instead of qh / kh / vh (head_dim 64, vector path only; rows past the
// sequence are left to attn_img_pad_kernel).
int laya_prep(const char* op, const float* qkv, const float* cos_t, const float* sin_t,
              float* qh, float* kh, float* vh, int64_t hidden, int64_t heads, int64_t length,
              int64_t batch, cudaStream_t stream, uint8_t* flags = nullptr,
              uint8_t* const* img = nullptr, bool late = false) {
  TFX_REQUIRE(hidden >= 0 && heads > 0 && length >= 0 && batch >= 0, op, "shape",
              "extents must be non-negative (heads positive)");
  TFX_REQUIRE(hidden % heads == 0, op, "hidden", "hidden must be a multiple of heads");
  const int64_t hd = hidden / heads;
  TFX_REQUIRE(hd % 2 == 0, op, "head_dim", "head_dim must be even");
  if (hidden == 0 || length == 0 || batch == 0) return TFX_OK;
  TFX_REQUIRE(qkv && (img || (qh && kh && vh)), op, "tensors", "null pointer");
  TFX_REQUIRE((cos_t == nullptr) == (sin_t == nullptr), op, "tables",
              "cos and sin tables must both be given or both be null");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  const int64_t half = hd / 2;
  const bool v4 = half % 4 == 0 && hidden % 4 == 0 && aligned(qkv, 16) &&
                  (img || (aligned(qh, 16) && aligned(kh, 16) && aligned(vh, 16))) &&
                  (!cos_t || (aligned(cos_t, 16) && aligned(sin_t, 16)));
  if (img && !(v4 && hd == 64))
    return fail(TFX_ERR_UNSUPPORTED, op, "layout", "tile images need head_dim 64 and 16-byte rows");
  const int64_t vec = v4 ? 4 : 1;
  const int64_t chunks = half / vec;
  const int64_t total = batch * length * heads * chunks;
  TFX_REQUIRE(total < (int64_t(1) << 32) && batch * length < (int64_t(1) << 32), op, "shape",
              "too many elements for one call");
  const unsigned grid = unsigned(std::min<int64_t>((total + 255) / 256, 148 * 16));
  const FastDiv dc{uint32_t(chunks)}, dh{uint32_t(heads)}, dl{uint32_t(length)};
  uint8_t* const no_img = nullptr;
  if (img) {
    const uint32_t nqt = uint32_t((length + kWsTQ - 1) / kWsTQ);
    const uint32_t nkt = uint32_t((length + kWsKB - 1) / kWsKB);
    auto run = [&](auto kernel) {
      return launch_kernel(op, kernel, dim3(grid), dim3(256), 0, stream, 1, qkv, cos_t, sin_t,
                           qh, kh, vh, uint32_t(hidden), uint32_t(heads), uint32_t(length),
                           uint32_t(hd), uint64_t(total), dc, dh, dl, flags, img[0], img[1],
                           img[2], nqt, nkt);
    };
    return late ? run(laya_prep_kernel<4, true, true>) : run(laya_prep_kernel<4, true>);
  }
  if (v4)
    return launch_kernel(op, laya_prep_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, qkv, cos_t,
                         sin_t, qh, kh, vh, uint32_t(hidden), uint32_t(heads), uint32_t(length),
                         uint32_t(hd), uint64_t(total), dc, dh, dl, flags, no_img, no_img, no_img,
                         0u, 0u);
  return launch_kernel(op, laya_prep_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, qkv, cos_t,
                       sin_t, qh, kh, vh, uint32_t(hidden), uint32_t(heads), uint32_t(length),
                       uint32_t(hd), uint64_t(total), dc, dh, dl, flags, no_img, no_img, no_img,
                       0u, 0u);
}

int jeff_prep(const char* op, const float* q, const float* k, const float* v,
              const float* q_norm, const float* k_norm, const float* cos_t, const float* sin_t,
              float* qh, float* kh, float* vh, int64_t length, int64_t heads, int64_t head_dim,
              int64_t rotary_dim, float eps, cudaStream_t stream) {
  TFX_REQUIRE(length >= 0 && heads >= 0 && head_dim >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0, op,
              "rotary_dim", "rotary_dim must be even and at most head_dim");
  TFX_REQUIRE(head_dim <= 1024, op, "head_dim", "head_dim above 1024");
  if (length == 0 || heads == 0 || head_dim == 0) return TFX_OK;
  TFX_REQUIRE(q && k && v && qh && kh && vh && q_norm && k_norm, op, "tensors", "null pointer");
  TFX_REQUIRE(rotary_dim == 0 || (cos_t && sin_t), op, "tables", "null pointer");
  TFX_REQUIRE(length < (int64_t(1) << 31) && heads < 65536, op, "shape", "too large");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  const size_t smem = size_t(head_dim) * 33 * 4;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(
        jeff_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(e));
  }
  return launch_kernel(op, jeff_prep_kernel, dim3(unsigned((length + 31) / 32), unsigned(heads)),
                       dim3(256), smem, stream, 1, q, k, v, q_norm, k_norm, cos_t, sin_t, qh, kh,
                       vh, uint32_t(length), uint32_t(head_dim), uint32_t(rotary_dim), eps);
}

// img (optional, head_dim 64 with attn_tc_covers): q, k, v as tile images
// instead of qh / kh / vh.
AttnArgs attn_args(const float* qh, const float* kh, const float* vh, float* out,
                   const tfx_attention_desc* d);

// digest_words / digest_summary (optional): the keep / active digest,
// computed before the call.
int attention(const char* op, const float* qh, const float* kh, const float* vh, float* out,
              const tfx_attention_desc* d, cudaStream_t stream,
              const uint8_t* pre_flags = nullptr, uint8_t* const* img = nullptr,
              const uint32_t* digest_words = nullptr, const uint8_t* digest_summary = nullptr) {
  TFX_REQUIRE(d, op, "desc", "null pointer");
  TFX_REQUIRE(d->batch >= 0 && d->heads >= 0 && d->length >= 0 && d->head_dim >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(d->empty_rows == TFX_ATTN_EMPTY_NAN || d->empty_rows == TFX_ATTN_EMPTY_ZERO, op,
              "empty_rows", "unknown value " + std::to_string(d->empty_rows));
  if (d->batch == 0 || d->heads == 0 || d->length == 0 || d->head_dim == 0) return TFX_OK;
  TFX_REQUIRE((img || (qh && kh && vh)) && out, op, "tensors", "null pointer");
  TFX_REQUIRE(d->length < (int64_t(1) << 31) && d->heads < 65536 && d->batch < 65536, op,
              "shape", "too large");
  TFX_REQUIRE(d->head_dim <= 1024, op, "head_dim", "head_dim above 1024");
  AttnArgs a = attn_args(qh, kh, vh, out, d);
  if (img) {
    a.qimg = img[0];
    a.kimg = img[1];
    a.vimg = img[2];
    a.nqt = uint32_t((d->length + kWsTQ - 1) / kWsTQ);
    a.nkt = uint32_t((d->length + kWsKB - 1) / kWsKB);
  }
  a.digest_words = digest_words;
  a.digest_summary = digest_summary;
  return attn_launch(op, a, uint32_t(d->batch), stream, pre_flags);
}

// The Jeff attention descriptor (fused.cu / lib.rs Jeff path): causal over the
// active keys, empty rows 0, gated, out (hidden, length).
tfx_attention_desc jeff_desc(const float* gate, const float* mask, int64_t length, int64_t heads,
                             int64_t head_dim) {
  tfx_attention_desc d;
  tfx_attention_desc_init(&d, 1, heads, length, head_dim);
  d.empty_rows = TFX_ATTN_EMPTY_ZERO;
  d.causal = 1;
  d.active = mask;
  d.gate = gate;
  d.out_tok = 1;
  d.out_feat = length;
  d.out_batch = 0;
  return d;
}

// The Jeff block on the tensor cores (length % 128 == 0, head_dim % 32 == 0):
// prep -> S_h = Q_h K_h^T -> causal / active softmax in place -> V_h^T ->
// O_h = P_h V_h -> gate into (hidden, length); heads that prep flagged are
// then redone by the f32 kernel. qkv: the 3 n floats of head-major scratch.
int jeff_attention_tc(const char* op, const float* q, const float* k, const float* v,
                      const float* gate, const float* q_norm, const float* k_norm,
                      const float* mask, const float* cos_t, const float* sin_t, float* out,
                      int64_t length, int64_t heads, int64_t head_dim, int64_t rotary_dim,
                      float eps, cudaStream_t s) {
  const int64_t n = length * heads * head_dim;
  const int64_t nscore = heads * length * length;
  CausalKSplit split;
  int rc = gemm_causal_k_split(heads * length, length, &split);
  if (rc != TFX_OK) return rc;
  const uint32_t slots = split.max_pieces(uint32_t(heads));
  // scratch (floats): q hi | q lo | k hi | k lo | V^T hi | V^T lo | scores |
  // P hi | P lo | O slots, then keep bytes | first active key | flags
  const size_t floats = size_t(6 * n + 3 * nscore + int64_t(slots) * n);
  const size_t keep_off = floats * 4;
  const size_t first_off = keep_off + (size_t(length) + 255) / 256 * 256;
  const size_t flags_off = first_off + 256;
  uint8_t* work = nullptr;
  cudaError_t e = scratch_malloc(reinterpret_cast<void**>(&work),
                                 flags_off + (size_t(heads) + 255) / 256 * 256, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  }
  float* f = reinterpret_cast<float*>(work);
  float* qhi = f;
  float* qlo = f + n;
  float* khi = f + 2 * n;
  float* klo = f + 3 * n;
  float* vthi = f + 4 * n;
  float* vtlo = f + 5 * n;
  float* scores = f + 6 * n;
  float* phi = scores + nscore;
  float* plo = phi + nscore;
  float* o = plo + nscore;
  uint8_t* keep = work + keep_off;
  int* first = reinterpret_cast<int*>(work + first_off);
  uint8_t* flags = work + flags_off;
  const uint32_t L = uint32_t(length), hd = uint32_t(head_dim), H = uint32_t(heads);
  e = cudaMemsetAsync(first, 0x7F, 4, s);  // 0x7F7F7F7F: no active key yet
  if (e == cudaSuccess) e = cudaMemsetAsync(flags, 0, size_t(heads), s);
  if (e != cudaSuccess) rc = fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  if (rc == TFX_OK) {
    const dim3 grid(L / 32, H, 3);
    auto prep = [&](auto kernel) {
      return launch_kernel(op, kernel, grid, dim3(256), 0, s, 1, q, k, v, q_norm, k_norm, cos_t,
                           sin_t, qhi, qlo, khi, klo, vthi, vtlo, L, uint32_t(rotary_dim), eps,
                           flags);
    };
    rc = hd == 256   ? prep(jeff_prep_planes_kernel<256>)
         : hd == 128 ? prep(jeff_prep_planes_kernel<128>)
                     : prep(jeff_prep_planes_kernel<64>);
  }
  if (rc == TFX_OK)
    rc = launch_kernel(op, jeff_keep_kernel, dim3(std::min<uint32_t>((L + 255) / 256, 148)),
                       dim3(256), 0, s, 1, mask, keep, first, L);
  // S = Q K^T per head; scores above the diagonal's 256-key tiles are never
  // read and left unwritten
  if (rc == TFX_OK) {
    const float* planes[4] = {qhi, qlo, khi, klo};
    rc = gemm_batched_f32(op, nullptr, nullptr, scores, head_dim, length, heads * length, length,
                          s, 1, planes);
  }
  if (rc == TFX_OK) {
    const uint32_t rows = H * L;
    rc = launch_kernel(op, jeff_softmax_planes_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, 1,
                       static_cast<const float*>(scores), static_cast<const uint8_t*>(keep),
                       static_cast<const int*>(first), phi, plo, L, rows,
                       1.0f / sqrtf(float(head_dim)), split.row_tokens);
  }
  // O = P V per head, written (head, channel, token) into the split's slots
  if (rc == TFX_OK) {
    const float* planes[4] = {phi, plo, vthi, vtlo};
    rc = gemm_batched_f32(op, nullptr, nullptr, o, length, head_dim, heads * length, length, s, 2,
                          planes, 1);
  }
  if (rc == TFX_OK) {
    int st = TFX_OK;
    const DeviceInfo& dev = device_info(&st);
    if (st != TFX_OK) rc = st;
    const uint32_t nwarps = uint32_t(n / 128);  // n < 2^32: H L <= 2^23, hd <= 256
    const unsigned grid = std::min<unsigned>((nwarps + 7) / 8, unsigned(dev.sms) * 16);
    if (rc == TFX_OK)
      rc = launch_kernel(op, jeff_gate_kernel, dim3(grid), dim3(256), 0, s, 1,
                         static_cast<const float*>(o), gate, out, static_cast<const int*>(first),
                         uint64_t(n), L, hd, nwarps, split);
  }
  if (rc == TFX_OK) {
    // flagged heads: the f32 kernel (q, k as hi + lo, v from the V^T planes),
    // which returns at once for the others
    const tfx_attention_desc d = jeff_desc(gate, mask, length, heads, head_dim);
    AttnArgs a = attn_args(qhi, khi, vthi, out, &d);
    a.q_lo = qlo;
    a.k_lo = klo;
    a.v_lo = vtlo;
    a.vflags = flags;
    a.vflag_mode = 2;
    rc = attn_launch(op, a, 1, s, nullptr, true);
  }
  cudaFreeAsync(work, s);
  return rc;
}

AttnArgs attn_args(const float* qh, const float* kh, const float* vh, float* out,
                   const tfx_attention_desc* d) {
  AttnArgs a;
  a.q = qh;
  a.k = kh;
  a.v = vh;
  a.out = out;
  a.keep = d->keep;
  a.bias = d->bias;
  a.active = d->active;
  a.gate = d->gate;
  a.gate_offset = d->gate_offset;
  a.out_tok = d->out_tok;
  a.out_feat = d->out_feat;
  a.out_batch = d->out_batch;
  a.heads = uint32_t(d->heads);
  a.length = uint32_t(d->length);
  a.hd = uint32_t(d->head_dim);
  a.scale = d->scale;
  a.empty_nan = d->empty_rows == TFX_ATTN_EMPTY_NAN;
  a.causal = d->causal ? 1 : 0;
  a.window = d->window;
  a.valid_len = d->valid_len;
  a.vflags = nullptr;
  a.vflag_mode = 0;
  return a;
}

}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_rope_tables_powf_f32(float base, int64_t seq, int64_t rotary_dim, float* cos_host,
                             float* sin_host) {
  clear_error();
  const char* op = "cpu-kernels::rope_tables";
  TFX_REQUIRE(seq >= 0, op, "seq", "must be non-negative");
  TFX_REQUIRE(rotary_dim > 0 && rotary_dim % 2 == 0, op, "rotary_dim",
              "rotary width must be a positive even number, got " + std::to_string(rotary_dim));
  TFX_REQUIRE(seq == 0 || (cos_host && sin_host), op, "tables", "null pointer");
  const int64_t half = rotary_dim / 2;
  for (int64_t p = 0; p < seq; ++p)
    for (int64_t i = 0; i < half; ++i) {
      const float e = (-2.0f * float(i)) / float(rotary_dim);
      const float theta = float(p) * powf(base, e);
      cos_host[p * half + i] = cosf(theta);
      sin_host[p * half + i] = sinf(theta);
    }
  return TFX_OK;
}

int tfx_laya_qkv_prep_f32(const float* qkv, const float* cos_table, const float* sin_table,
                          float* qh, float* kh, float* vh, int64_t hidden, int64_t heads,
                          int64_t length, int64_t batch, tfx_stream_t stream) {
  clear_error();
  return laya_prep("tenferro-ext::laya_qkv_prep", qkv, cos_table, sin_table, qh, kh, vh, hidden,
                   heads, length, batch, static_cast<cudaStream_t>(stream));
}

int tfx_jeff_qkv_prep_f32(const float* q, const float* k, const float* v, const float* q_norm,
                          const float* k_norm, const float* cos_table, const float* sin_table,
                          float* qh, float* kh, float* vh, int64_t length, int64_t heads,
                          int64_t head_dim, int64_t rotary_dim, float eps, tfx_stream_t stream) {
  clear_error();
  return jeff_prep("tenferro-ext::jeff_qkv_prep", q, k, v, q_norm, k_norm, cos_table, sin_table,
                   qh, kh, vh, length, heads, head_dim, rotary_dim, eps,
                   static_cast<cudaStream_t>(stream));
}

int tfx_attention_desc_init(tfx_attention_desc* d, int64_t batch, int64_t heads, int64_t length,
                            int64_t head_dim) {
  clear_error();
  TFX_REQUIRE(d, "tenferro-ext::attention", "desc", "null pointer");
  *d = tfx_attention_desc{};
  d->batch = batch;
  d->heads = heads;
  d->length = length;
  d->head_dim = head_dim;
  d->scale = head_dim > 0 ? 1.0f / sqrtf(float(head_dim)) : 1.0f;
  d->empty_rows = TFX_ATTN_EMPTY_NAN;
  d->window = -1;
  d->valid_len = -1;
  d->out_tok = heads * head_dim;
  d->out_feat = 1;
  d->out_batch = heads * head_dim * length;
  return TFX_OK;
}

int tfx_attention_f32(const float* qh, const float* kh, const float* vh, float* out,
                      const tfx_attention_desc* desc, tfx_stream_t stream) {
  clear_error();
  return attention("tenferro-ext::attention", qh, kh, vh, out, desc,
                   static_cast<cudaStream_t>(stream));
}

int tfx_laya_attention_block_f32(const float* qkv, const uint8_t* keep, const float* cos_table,
                                 const float* sin_table, float* out, int64_t hidden,
                                 int64_t heads, int64_t length, int64_t batch,
                                 tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-ext::laya_attention_block";
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  TFX_REQUIRE(heads > 0 && hidden >= 0 && length >= 0 && batch >= 0, op, "shape",
              "extents must be non-negative (heads positive)");
  TFX_REQUIRE(hidden % heads == 0, op, "hidden", "hidden must be a multiple of heads");
  const int64_t n = hidden * length * batch;
  if (n == 0) return TFX_OK;
  TFX_REQUIRE(qkv && keep && out, op, "tensors", "null pointer");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  const int64_t hd = hidden / heads;
  const size_t nbh = size_t(batch * heads);
  const DeviceInfo& dev = device_info(&st);
  // head_dim 64 on the tensor cores: the prep kernel writes the attention's
  // tile images directly (hi / lo, 512 bytes per padded row and tensor);
  // otherwise head-major q, k, v. Then one flag byte per head (heads the
  // tensor-core attention leaves to the f32 one).
  const bool img = hd == 64 && aligned(qkv, 16) &&
                   (!cos_table || (aligned(cos_table, 16) && aligned(sin_table, 16))) &&
                   attn_tc_covers(64, uint64_t(n / hd), dev);
  const uint64_t lq = uint64_t((length + kWsTQ - 1) / kWsTQ) * kWsTQ;
  const uint64_t lk = uint64_t((length + kWsKB - 1) / kWsKB) * kWsKB;
  const size_t data_bytes = img ? nbh * (lq + 2 * lk) * 512 : size_t(3 * n) * 4;
  // with the images, the keep digest (1 KB of words and a summary byte per
  // (batch, query tile, key tile)) is computed first, overlapping the prep
  const uint32_t nqt = uint32_t(lq / kWsTQ), nkt = uint32_t(lk / kWsKB);
  const size_t dtiles = img ? size_t(batch) * nqt * nkt : 0;
  const size_t words_bytes = dtiles * 1024, summary_bytes = (dtiles + 255) / 256 * 256;
  uint8_t* scratch = nullptr;
  cudaError_t e = scratch_malloc(reinterpret_cast<void**>(&scratch),
                                 data_bytes + words_bytes + summary_bytes + nbh, s);
  uint32_t* words = reinterpret_cast<uint32_t*>(scratch + data_bytes);
  uint8_t* summary = scratch + data_bytes + words_bytes;
  uint8_t* flags = summary + summary_bytes;
  if (e == cudaSuccess) e = cudaMemsetAsync(flags, 0, nbh, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  }
  tfx_attention_desc d;
  tfx_attention_desc_init(&d, batch, heads, length, hd);
  d.keep = keep;
  float* raw = reinterpret_cast<float*>(scratch);
  uint8_t* const images[3] = {scratch, scratch + nbh * lq * 512, scratch + nbh * (lq + lk) * 512};
  int rc = TFX_OK;
  if (img)
    rc = launch_kernel(op, attn_keep_digest_kernel, dim3(nkt, nqt, unsigned(batch)), dim3(32), 0,
                       s, 1, attn_args(nullptr, nullptr, nullptr, out, &d), nqt, nkt, words,
                       summary);
  if (rc == TFX_OK)
    rc = img ? laya_prep(op, qkv, cos_table, sin_table, nullptr, nullptr, nullptr, hidden, heads,
                         length, batch, s, flags, images, /*late=*/true)
             : laya_prep(op, qkv, cos_table, sin_table, raw, raw + n, raw + 2 * n, hidden,
                         heads, length, batch, s, flags);
  if (rc == TFX_OK && img && lq != uint64_t(length)) {  // rows past the sequence: 0
    const uint64_t total = nbh * (lq - uint64_t(length)) * 16;
    rc = launch_kernel(op, attn_img_pad_kernel, dim3(unsigned(std::min<uint64_t>(
                                                     (total + 255) / 256, uint64_t(dev.sms) * 8))),
                       dim3(256), 0, s, 1, images[0], images[1], images[2], uint32_t(length),
                       uint32_t(lq), uint32_t(lk), total);
  }
  if (rc == TFX_OK)
    rc = img ? attention(op, nullptr, nullptr, nullptr, out, &d, s, flags, images, words, summary)
             : attention(op, raw, raw + n, raw + 2 * n, out, &d, s, flags);
  cudaFreeAsync(scratch, s);
  return rc;
}

int tfx_jeff_attention_f32(const float* q, const float* k, const float* v, const float* gate,
                           const float* q_norm, const float* k_norm, const float* mask,
                           const float* cos_table, const float* sin_table, float* out,
                           int64_t length, int64_t heads, int64_t head_dim, int64_t rotary_dim,
                           float eps, tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-ext::jeff_attention";
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  TFX_REQUIRE(length >= 0 && heads >= 0 && head_dim >= 0, op, "shape",
              "extents must be non-negative");
  const int64_t n = length * heads * head_dim;
  if (n == 0) return TFX_OK;
  TFX_REQUIRE(gate && mask && out, op, "tensors", "null pointer");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  // Tensor-core route (score GEMM, masked softmax, P V GEMM): whole 128-token
  // tiles, head_dim 64, 128 or 256 (one GEMM tile), scores of at most 2^30
  // values, 16-byte aligned gate and out. The prep checks come first.
  const bool tc = !attn_f32_only() && length % 128 == 0 &&
                  (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
                  heads * length * length <= (int64_t(1) << 30) && aligned(gate, 16) &&
                  aligned(out, 16);
  if (tc) {
    TFX_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0, op,
                "rotary_dim", "rotary_dim must be even and at most head_dim");
    TFX_REQUIRE(q && k && v && q_norm && k_norm, op, "tensors", "null pointer");
    TFX_REQUIRE(rotary_dim == 0 || (cos_table && sin_table), op, "tables", "null pointer");
    TFX_REQUIRE(heads < 65536, op, "shape", "too large");
    return jeff_attention_tc(op, q, k, v, gate, q_norm, k_norm, mask, cos_table, sin_table, out,
                             length, heads, head_dim, rotary_dim, eps, s);
  }
  float* scratch = nullptr;
  const cudaError_t e = scratch_malloc(reinterpret_cast<void**>(&scratch), size_t(3 * n) * 4, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  }
  int rc = jeff_prep(op, q, k, v, q_norm, k_norm, cos_table, sin_table, scratch, scratch + n,
                     scratch + 2 * n, length, heads, head_dim, rotary_dim, eps, s);
  if (rc == TFX_OK) {
    const tfx_attention_desc d = jeff_desc(gate, mask, length, heads, head_dim);
    rc = attention(op, scratch, scratch + n, scratch + 2 * n, out, &d, s);
  }
  cudaFreeAsync(scratch, s);
  return rc;
}

}  // extern "C"
