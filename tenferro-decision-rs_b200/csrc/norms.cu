// norms.cu -- feature-first LayerNorm and feature-last RMSNorm.
//
// LayerNorm (x is (d, cols), column c contiguous): one warp owns one column.
// The whole column is loaded into registers with 128-bit loads (d <= 1024 f32
// or d <= 1024 f64), so the reference's two passes -- the sum, then the
// centred sum of squares (crates/cpu-kernels/src/lib.rs:413-433) -- run over
// registers, and HBM sees exactly one read and one write of the activation.
// Wider columns use a CTA per column with the column held by 256 threads;
// anything else (unaligned, very wide) a CTA-per-column kernel that re-reads
// the column from L2.
//
// RMSNorm (x is column-major (rows, width): a token's features are strided by
// `rows`): a tile of 32*VEC consecutive tokens is read as one contiguous
// 128*VEC-byte run per feature, and the feature axis of the tile is split
// over a thread-block cluster of up to 8 CTAs. Each CTA keeps its share of the
// tile in registers, reduces its partial sums of squares per token in shared
// memory, and the cluster adds the partials through distributed shared memory
// before every CTA scales and writes its own share -- one read and one write
// of the activation, with the per-token reduction spread over up to 8 SMs.

#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace cg = cooperative_groups;

namespace tfx {
namespace {

// ---- arithmetic in the reference's operation order ------------------------------

template <typename T>
__device__ __forceinline__ T add_rn(T a, T b) {
  if constexpr (std::is_same_v<T, float>) return __fadd_rn(a, b);
  else return __dadd_rn(a, b);
}
template <typename T>
__device__ __forceinline__ T sub_rn(T a, T b) {
  if constexpr (std::is_same_v<T, float>) return __fsub_rn(a, b);
  else return __dsub_rn(a, b);
}
template <typename T>
__device__ __forceinline__ T mul_rn(T a, T b) {
  if constexpr (std::is_same_v<T, float>) return __fmul_rn(a, b);
  else return __dmul_rn(a, b);
}
template <typename T>
__device__ __forceinline__ T div_rn(T a, T b) {
  if constexpr (std::is_same_v<T, float>) return __fdiv_rn(a, b);
  else return __ddiv_rn(a, b);
}
template <typename T>
__device__ __forceinline__ T sqrt_rn(T a) {
  if constexpr (std::is_same_v<T, float>) return __fsqrt_rn(a);
  else return __dsqrt_rn(a);
}

// f32 (cpu-kernels lib.rs:413-424) divides the sums by d; the f64 composite
// (tenferro-infer norm.rs:23-30) multiplies them by 1/width.
template <typename T>
__device__ __forceinline__ T scale_by_width(T sum, T d, T inv_d) {
  if constexpr (std::is_same_v<T, float>) return div_rn(sum, d);
  else return mul_rn(sum, inv_d);
}

// 16-byte vector of T.
template <typename T>
struct V16;
template <>
struct V16<float> {
  static constexpr int N = 4;
  float v[4];
};
template <>
struct V16<double> {
  static constexpr int N = 2;
  double v[2];
};

template <typename T>
__device__ __forceinline__ V16<T> load16(const T* p) {
  V16<T> r;
  if constexpr (std::is_same_v<T, float>) {
    const float4 q = ld_stream(reinterpret_cast<const float4*>(p));
    r.v[0] = q.x; r.v[1] = q.y; r.v[2] = q.z; r.v[3] = q.w;
  } else {
    const double2 q = ld_stream(reinterpret_cast<const double2*>(p));
    r.v[0] = q.x; r.v[1] = q.y;
  }
  return r;
}
template <typename T>
__device__ __forceinline__ V16<T> ldg16(const T* p) {
  V16<T> r;
  if constexpr (std::is_same_v<T, float>) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(p));
    r.v[0] = q.x; r.v[1] = q.y; r.v[2] = q.z; r.v[3] = q.w;
  } else {
    const double2 q = __ldg(reinterpret_cast<const double2*>(p));
    r.v[0] = q.x; r.v[1] = q.y;
  }
  return r;
}
template <typename T>
__device__ __forceinline__ void store16(T* p, const V16<T>& r) {
  if constexpr (std::is_same_v<T, float>)
    *reinterpret_cast<float4*>(p) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
  else
    *reinterpret_cast<double2*>(p) = make_double2(r.v[0], r.v[1]);
}

template <typename T>
__device__ __forceinline__ T warp_sum_t(T v) {
  return warp_sum(v);
}

// ---- LayerNorm: one warp per column, column in registers --------------------------

// NV = 16-byte vectors per lane; d <= 32 * NV * V16<T>::N and d % V16<T>::N == 0.
template <typename T, int NV, bool BIAS>
__global__ void __launch_bounds__(256) ln_warp_kernel(const T* __restrict__ x,
                                                      const T* __restrict__ w,
                                                      const T* __restrict__ b, T* __restrict__ y,
                                                      uint32_t d, uint64_t cols, T eps) {
  pdl_enter();
  constexpr int VN = V16<T>::N;
  const int lane = threadIdx.x & 31;
  const uint64_t col = uint64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (col >= cols) return;  // the whole warp leaves together
  const uint32_t dv = d / VN;
  const T* xc = x + col * d;
  V16<T> v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) v[j] = load16(xc + q * VN);
  }
  T s = T(0);
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (j * 32 + lane < dv)
#pragma unroll
      for (int k = 0; k < VN; ++k) s = add_rn(s, v[j].v[k]);
  s = warp_sum_t(s);
  const T dd = T(d), inv_d = T(1) / T(d);
  const T mean = scale_by_width(s, dd, inv_d);
  T ss = T(0);
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (j * 32 + lane < dv)
#pragma unroll
      for (int k = 0; k < VN; ++k) {
        const T c = sub_rn(v[j].v[k], mean);
        ss = add_rn(ss, mul_rn(c, c));
      }
  ss = warp_sum_t(ss);
  const T var = scale_by_width(ss, dd, inv_d);
  const T inv = div_rn(T(1), sqrt_rn(add_rn(var, eps)));
  T* yc = y + col * d;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const V16<T> wv = ldg16(w + q * VN);
      V16<T> o;
#pragma unroll
      for (int k = 0; k < VN; ++k) o.v[k] = mul_rn(mul_rn(sub_rn(v[j].v[k], mean), inv), wv.v[k]);
      if constexpr (BIAS) {
        const V16<T> bv = ldg16(b + q * VN);
#pragma unroll
        for (int k = 0; k < VN; ++k) o.v[k] = add_rn(o.v[k], bv.v[k]);
      }
      store16(yc + q * VN, o);
    }
  }
}

// ---- LayerNorm f32: one warp per column, column staged in shared memory ------------
//
// Same arithmetic as ln_warp_kernel, but the column is copied into the warp's
// slice of shared memory with cp.async (16 bytes per lane per step) instead of
// being held in registers. At 32 registers per thread 64 warps fit on an SM,
// so 148 SMs keep 9472 columns in flight at once -- config-sized tensors
// (8192 columns of 768) run in a single wave instead of 1.4.

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

template <int NV, bool BIAS>
__global__ void __launch_bounds__(256, 8) ln_smem_kernel(const float* __restrict__ x,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ b,
                                                         float* __restrict__ y, uint32_t d,
                                                         uint64_t cols, float eps) {
  pdl_enter();
  extern __shared__ float4 stage[];  // 8 warps x d floats
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t col = uint64_t(blockIdx.x) * 8 + warp;
  if (col >= cols) return;  // the whole warp leaves together
  const uint32_t dv = d / 4;
  float4* sx = stage + warp * dv;
  const float4* xc = reinterpret_cast<const float4*>(x + col * d);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) cp_async16(sx + q, xc + q);
  }
  cp_async_wait_all();
  __syncwarp();
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const float4 v = sx[q];
      s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v.x), v.y), v.z), v.w);
    }
  }
  s = warp_sum(s);
  const float dd = float(d);
  const float mean = __fdiv_rn(s, dd);
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const float4 v = sx[q];
      const float cx = __fsub_rn(v.x, mean), cy = __fsub_rn(v.y, mean);
      const float cz = __fsub_rn(v.z, mean), cw = __fsub_rn(v.w, mean);
      ss = __fadd_rn(ss, __fmul_rn(cx, cx));
      ss = __fadd_rn(ss, __fmul_rn(cy, cy));
      ss = __fadd_rn(ss, __fmul_rn(cz, cz));
      ss = __fadd_rn(ss, __fmul_rn(cw, cw));
    }
  }
  ss = warp_sum(ss);
  const float var = __fdiv_rn(ss, dd);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  float4* yc = reinterpret_cast<float4*>(y + col * d);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const float4 v = sx[q];
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
      float4 o;
      o.x = __fmul_rn(__fmul_rn(__fsub_rn(v.x, mean), inv), wv.x);
      o.y = __fmul_rn(__fmul_rn(__fsub_rn(v.y, mean), inv), wv.y);
      o.z = __fmul_rn(__fmul_rn(__fsub_rn(v.z, mean), inv), wv.z);
      o.w = __fmul_rn(__fmul_rn(__fsub_rn(v.w, mean), inv), wv.w);
      if constexpr (BIAS) {
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b) + q);
        o.x = __fadd_rn(o.x, bv.x);
        o.y = __fadd_rn(o.y, bv.y);
        o.z = __fadd_rn(o.z, bv.z);
        o.w = __fadd_rn(o.w, bv.w);
      }
      yc[q] = o;
    }
  }
}

// ---- LayerNorm f32: persistent warps, each with a ring of column slots -------------
//
// One CTA of 16 warps per SM; warp g of G handles columns g, g + G, g + 2G, ...
// Each warp owns LN_RING_SLOTS shared-memory slots of one column: while it
// reduces and writes column k from its slot, cp.async copies columns k+1 and
// k+2 into the other two, so every SM keeps 32 columns (96 KB at d = 768) in
// flight and each column's arithmetic and store overlap later columns' loads.
// The weights (and bias) are read once per warp into registers instead of once
// per column. The lane -> element mapping and every rounding are those of
// ln_smem_kernel, so the two kernels give identical bits.
//
// Why not one column per warp in a single wave (ln_smem_kernel): all 8192
// columns of configs[0] request their reads at once, the memory system serves
// them interleaved, most columns complete only near the end of the read
// phase, and the arithmetic, the weight loads and the writes of nearly every
// column then fall into the last microseconds. Measured on configs[0] (CUDA
// graph of 40 launches over rotating buffers, no programmatic launch): 9.56 us
// for this kernel, 9.96 us for ln_smem_kernel, 9.14 us for a copy of the same
// bytes with the same warp-per-column tiling; 8 warps x 2 CTAs, 12 or 20
// warps, 2 or 4 slots, and register double buffering instead of shared memory
// all measured 9.5 - 10.3 us. With many columns per warp the ring loses (the
// dispatcher below picks by column count).
constexpr int LN_RING_WARPS = 16;
constexpr int LN_RING_SLOTS = 3;

template <int NV, bool BIAS>
__global__ void __launch_bounds__(LN_RING_WARPS * 32, 1) ln_ring_kernel(
    const float* x, const float* __restrict__ w, const float* __restrict__ b, float* y,
    uint32_t d, uint64_t cols, float eps) {
  pdl_enter();
  extern __shared__ float4 stage[];  // LN_RING_WARPS x LN_RING_SLOTS x d floats
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t gw = uint64_t(blockIdx.x) * LN_RING_WARPS + warp;
  const uint64_t G = uint64_t(gridDim.x) * LN_RING_WARPS;
  const uint32_t dv = d / 4;
  if (gw >= cols) return;  // the whole warp leaves together
  float4 wr[NV], br[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      wr[j] = __ldg(reinterpret_cast<const float4*>(w) + q);
      if constexpr (BIAS) br[j] = __ldg(reinterpret_cast<const float4*>(b) + q);
    }
  }
  float4* ring = stage + size_t(warp) * LN_RING_SLOTS * dv;
  const uint64_t n = (cols - gw + G - 1) / G;  // columns of this warp
  // Copies column k of this warp into slot k % LN_RING_SLOTS as one cp.async
  // group (an empty group past the last column keeps the group count uniform).
  auto issue = [&](uint64_t k) {
    if (k < n) {
      const float4* xc = reinterpret_cast<const float4*>(x + (gw + k * G) * d);
      float4* sl = ring + (k % LN_RING_SLOTS) * dv;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const uint32_t q = j * 32 + lane;
        if (q < dv) cp_async16(sl + q, xc + q);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
#pragma unroll
  for (int k = 0; k < LN_RING_SLOTS - 1; ++k) issue(k);
  const float dd = float(d);
  for (uint64_t k = 0; k < n; ++k) {
    issue(k + LN_RING_SLOTS - 1);
    // groups complete in order: all but the newest LN_RING_SLOTS - 1 are done
    asm volatile("cp.async.wait_group %0;" ::"n"(LN_RING_SLOTS - 1) : "memory");
    __syncwarp();
    const float4* sl = ring + (k % LN_RING_SLOTS) * dv;
    float4 v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const uint32_t q = j * 32 + lane;
      if (q < dv) v[j] = sl[q];
    }
    // every lane has read the slot before any lane's next issue overwrites it
    __syncwarp();
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (j * 32 + lane < dv)
        s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[j].x), v[j].y), v[j].z), v[j].w);
    s = warp_sum(s);
    const float mean = __fdiv_rn(s, dd);
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
      if (j * 32 + lane < dv) {
        const float cx = __fsub_rn(v[j].x, mean), cy = __fsub_rn(v[j].y, mean);
        const float cz = __fsub_rn(v[j].z, mean), cw = __fsub_rn(v[j].w, mean);
        ss = __fadd_rn(ss, __fmul_rn(cx, cx));
        ss = __fadd_rn(ss, __fmul_rn(cy, cy));
        ss = __fadd_rn(ss, __fmul_rn(cz, cz));
        ss = __fadd_rn(ss, __fmul_rn(cw, cw));
      }
    ss = warp_sum(ss);
    const float var = __fdiv_rn(ss, dd);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    float4* yc = reinterpret_cast<float4*>(y + (gw + k * G) * d);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const uint32_t q = j * 32 + lane;
      if (q < dv) {
        float4 o;
        o.x = __fmul_rn(__fmul_rn(__fsub_rn(v[j].x, mean), inv), wr[j].x);
        o.y = __fmul_rn(__fmul_rn(__fsub_rn(v[j].y, mean), inv), wr[j].y);
        o.z = __fmul_rn(__fmul_rn(__fsub_rn(v[j].z, mean), inv), wr[j].z);
        o.w = __fmul_rn(__fmul_rn(__fsub_rn(v[j].w, mean), inv), wr[j].w);
        if constexpr (BIAS) {
          o.x = __fadd_rn(o.x, br[j].x);
          o.y = __fadd_rn(o.y, br[j].y);
          o.z = __fadd_rn(o.z, br[j].z);
          o.w = __fadd_rn(o.w, br[j].w);
        }
        yc[q] = o;
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---- residual add fused into the LayerNorm that follows it ----------------------------
//
// s = a + b per element, then ln_smem_kernel's arithmetic on s (same order of
// every rounding), so y is bit-identical to tfx_add_f32 followed by
// tfx_layernorm_ff_f32; s is also written when SUM. Both inputs are staged
// with cp.async (two column slices per warp), so the sum never round-trips
// through HBM before the normalisation reads it.
template <int NV, bool BIAS, bool SUM>
__global__ void __launch_bounds__(256, 4) add_ln_smem_kernel(
    const float* __restrict__ a, const float* __restrict__ bsrc, const float* __restrict__ w,
    const float* __restrict__ b, float* sum_out, float* y, uint32_t d, uint64_t cols, float eps) {
  pdl_enter();
  extern __shared__ float4 stage[];  // 8 warps x 2 x d floats
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t col = uint64_t(blockIdx.x) * 8 + warp;
  if (col >= cols) return;  // the whole warp leaves together
  const uint32_t dv = d / 4;
  float4* sx = stage + warp * 2 * dv;
  float4* sb = sx + dv;
  const float4* ac = reinterpret_cast<const float4*>(a + col * d);
  const float4* bc = reinterpret_cast<const float4*>(bsrc + col * d);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      cp_async16(sx + q, ac + q);
      cp_async16(sb + q, bc + q);
    }
  }
  cp_async_wait_all();
  __syncwarp();
  float4* sc = reinterpret_cast<float4*>(sum_out + col * d);
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const float4 u = sx[q], t = sb[q];
      const float4 v = make_float4(__fadd_rn(u.x, t.x), __fadd_rn(u.y, t.y), __fadd_rn(u.z, t.z),
                                   __fadd_rn(u.w, t.w));
      sx[q] = v;
      if constexpr (SUM) sc[q] = v;
      s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v.x), v.y), v.z), v.w);
    }
  }
  s = warp_sum(s);
  const float dd = float(d);
  const float mean = __fdiv_rn(s, dd);
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const float4 v = sx[q];
      const float cx = __fsub_rn(v.x, mean), cy = __fsub_rn(v.y, mean);
      const float cz = __fsub_rn(v.z, mean), cw = __fsub_rn(v.w, mean);
      ss = __fadd_rn(ss, __fmul_rn(cx, cx));
      ss = __fadd_rn(ss, __fmul_rn(cy, cy));
      ss = __fadd_rn(ss, __fmul_rn(cz, cz));
      ss = __fadd_rn(ss, __fmul_rn(cw, cw));
    }
  }
  ss = warp_sum(ss);
  const float var = __fdiv_rn(ss, dd);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  float4* yc = reinterpret_cast<float4*>(y + col * d);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 32 + lane;
    if (q < dv) {
      const float4 v = sx[q];
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + q);
      float4 o;
      o.x = __fmul_rn(__fmul_rn(__fsub_rn(v.x, mean), inv), wv.x);
      o.y = __fmul_rn(__fmul_rn(__fsub_rn(v.y, mean), inv), wv.y);
      o.z = __fmul_rn(__fmul_rn(__fsub_rn(v.z, mean), inv), wv.z);
      o.w = __fmul_rn(__fmul_rn(__fsub_rn(v.w, mean), inv), wv.w);
      if constexpr (BIAS) {
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b) + q);
        o.x = __fadd_rn(o.x, bv.x);
        o.y = __fadd_rn(o.y, bv.y);
        o.z = __fadd_rn(o.z, bv.z);
        o.w = __fadd_rn(o.w, bv.w);
      }
      yc[q] = o;
    }
  }
}

// ---- LayerNorm: one CTA (256 threads) per column, column in registers --------------

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red /* [8] */) {
  v = warp_sum_t(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // red may still be read from a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T s = T(0);
#pragma unroll
  for (int i = 0; i < 8; ++i) s = add_rn(s, red[i]);
  return s;
}

template <typename T, int NV, bool BIAS>
__global__ void __launch_bounds__(256) ln_cta_kernel(const T* __restrict__ x,
                                                     const T* __restrict__ w,
                                                     const T* __restrict__ b, T* __restrict__ y,
                                                     uint32_t d, T eps) {
  pdl_enter();
  constexpr int VN = V16<T>::N;
  __shared__ T red[8];
  const uint64_t col = blockIdx.x;
  const uint32_t dv = d / VN;
  const T* xc = x + col * d;
  V16<T> v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 256 + threadIdx.x;
    if (q < dv) v[j] = load16(xc + q * VN);
  }
  T s = T(0);
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (j * 256 + threadIdx.x < dv)
#pragma unroll
      for (int k = 0; k < VN; ++k) s = add_rn(s, v[j].v[k]);
  s = block_sum(s, red);
  const T dd = T(d), inv_d = T(1) / T(d);
  const T mean = scale_by_width(s, dd, inv_d);
  T ss = T(0);
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (j * 256 + threadIdx.x < dv)
#pragma unroll
      for (int k = 0; k < VN; ++k) {
        const T c = sub_rn(v[j].v[k], mean);
        ss = add_rn(ss, mul_rn(c, c));
      }
  ss = block_sum(ss, red);
  const T var = scale_by_width(ss, dd, inv_d);
  const T inv = div_rn(T(1), sqrt_rn(add_rn(var, eps)));
  T* yc = y + col * d;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t q = j * 256 + threadIdx.x;
    if (q < dv) {
      const V16<T> wv = ldg16(w + q * VN);
      V16<T> o;
#pragma unroll
      for (int k = 0; k < VN; ++k) o.v[k] = mul_rn(mul_rn(sub_rn(v[j].v[k], mean), inv), wv.v[k]);
      if constexpr (BIAS) {
        const V16<T> bv = ldg16(b + q * VN);
#pragma unroll
        for (int k = 0; k < VN; ++k) o.v[k] = add_rn(o.v[k], bv.v[k]);
      }
      store16(yc + q * VN, o);
    }
  }
}

// ---- LayerNorm: any d, any alignment (three passes over the column, L2-resident) --

template <typename T>
__global__ void __launch_bounds__(256) ln_generic_kernel(const T* x, const T* __restrict__ w,
                                                         const T* __restrict__ b, T* y,
                                                         uint64_t d, T eps) {
  pdl_enter();
  __shared__ T red[8];
  const T* xc = x + uint64_t(blockIdx.x) * d;
  T* yc = y + uint64_t(blockIdx.x) * d;
  T s = T(0);
  for (uint64_t i = threadIdx.x; i < d; i += 256) s = add_rn(s, xc[i]);
  s = block_sum(s, red);
  const T dd = T(d), inv_d = T(1) / T(d);
  const T mean = scale_by_width(s, dd, inv_d);
  T ss = T(0);
  for (uint64_t i = threadIdx.x; i < d; i += 256) {
    const T c = sub_rn(xc[i], mean);
    ss = add_rn(ss, mul_rn(c, c));
  }
  ss = block_sum(ss, red);
  const T var = scale_by_width(ss, dd, inv_d);
  const T inv = div_rn(T(1), sqrt_rn(add_rn(var, eps)));
  for (uint64_t i = threadIdx.x; i < d; i += 256) {
    T o = mul_rn(mul_rn(sub_rn(xc[i], mean), inv), w[i]);
    if (b) o = add_rn(o, b[i]);
    yc[i] = o;
  }
}

// Launches ln_ring_kernel<NV, BIAS> on `grid` CTAs (at most one per SM),
// opting the instance in to the device's largest dynamic shared memory once
// per device.
template <int NV, bool BIAS>
int launch_ln_ring(const char* op, const DeviceInfo& dev, unsigned grid, size_t smem,
                   cudaStream_t stream, const float* x, const float* w, const float* b, float* y,
                   uint32_t d, uint64_t cols, float eps) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  const int di = dev.device & 63;
  std::call_once(once[di], [&] {
    err[di] = cudaFuncSetAttribute(ln_ring_kernel<NV, BIAS>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, dev.smem_optin);
  });
  if (err[di] != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(err[di]));
  return launch_kernel(op, ln_ring_kernel<NV, BIAS>, dim3(grid), dim3(LN_RING_WARPS * 32), smem,
                       stream, 1, x, w, b, y, d, cols, eps);
}

template <typename T>
int layernorm_ff(const char* op, const T* x, const T* w, const T* b, T* y, int64_t d,
                 int64_t cols, T eps, cudaStream_t stream) {
  clear_error();
  TFX_REQUIRE(d >= 0 && cols >= 0, op, "shape", "extents must be non-negative");
  if (d == 0 || cols == 0) return TFX_OK;
  TFX_REQUIRE(x, op, "x", "null pointer");
  TFX_REQUIRE(w, op, "weight", "null pointer");
  TFX_REQUIRE(y, op, "y", "null pointer");
  const size_t bytes = size_t(d) * size_t(cols) * sizeof(T);
  TFX_REQUIRE(y == x || !overlaps(x, bytes, y, bytes), op, "y", "partially overlaps x");
  TFX_REQUIRE(!overlaps(w, size_t(d) * sizeof(T), y, bytes), op, "weight", "overlaps y");
  TFX_REQUIRE(!b || !overlaps(b, size_t(d) * sizeof(T), y, bytes), op, "bias", "overlaps y");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  constexpr int VN = V16<T>::N;
  const bool vec = d % VN == 0 && aligned(x, 16) && aligned(y, 16) && aligned(w, 16) &&
                   (!b || aligned(b, 16));
  const int64_t dv = d / VN;
  const bool bias = b != nullptr;
  if constexpr (std::is_same_v<T, float>) {
    // Persistent ring kernel (f32, d <= 1024, up to ~5 columns per ring warp),
    // else the one-wave shared-memory kernel; TFX_LN_KERNEL=ring / smem / regs
    // forces one for tuning runs.
    static const int choice = [] {
      const char* e = getenv("TFX_LN_KERNEL");
      const std::string v = e ? e : "";
      return v == "regs" ? 2 : v == "smem" ? 1 : v == "ring" ? 3 : 0;
    }();
    const DeviceInfo& dev = device_info(&st);
    const size_t ring_smem = size_t(LN_RING_WARPS) * LN_RING_SLOTS * size_t(d) * 4;
    // The ring wins while each of its warps has few columns (configs[0]: 8192
    // columns, 3.5 per warp: 9.56 us against 9.96); with many columns per warp
    // its 16 warps per SM cannot hide each column's serial reductions and the
    // one-wave-per-64-warps kernel is faster (32768 columns: 32.2 us against
    // 35.7; equal at 16384).
    const bool ring_shape = cols <= int64_t(5) * dev.sms * LN_RING_WARPS;
    if (vec && dv <= 32 * 8 && ((choice == 0 && ring_shape) || choice == 3) &&
        ring_smem <= size_t(dev.smem_optin)) {
      const uint32_t du = uint32_t(d);
      const unsigned grid = unsigned(std::min<int64_t>(
          dev.sms, (cols + LN_RING_WARPS - 1) / LN_RING_WARPS));
#define TFX_LN_RING(NVV)                                                                     \
  if (dv <= 32 * NVV)                                                                        \
    return bias ? launch_ln_ring<NVV, true>(op, dev, grid, ring_smem, stream, x, w, b, y, du, \
                                            uint64_t(cols), eps)                             \
                : launch_ln_ring<NVV, false>(op, dev, grid, ring_smem, stream, x, w, b, y, du, \
                                             uint64_t(cols), eps);
      TFX_LN_RING(1)
      TFX_LN_RING(2)
      TFX_LN_RING(3)
      TFX_LN_RING(4)
      TFX_LN_RING(6)
      TFX_LN_RING(8)
#undef TFX_LN_RING
    }
    if (vec && dv <= 32 * 8 && choice != 2) {
      TFX_REQUIRE(cols / 8 < (int64_t(1) << 31), op, "cols", "too many columns for one call");
      const unsigned grid = unsigned((cols + 7) / 8);
      const uint32_t du = uint32_t(d);
      const size_t smem = size_t(8) * size_t(d) * 4;
#define TFX_LN_SMEM(NVV)                                                                       \
  if (dv <= 32 * NVV) {                                                                         \
    return bias ? launch_kernel(op, ln_smem_kernel<NVV, true>, dim3(grid), dim3(256), smem,      \
                                stream, 1, x, w, b, y, du, uint64_t(cols), eps)                  \
                : launch_kernel(op, ln_smem_kernel<NVV, false>, dim3(grid), dim3(256), smem,     \
                                stream, 1, x, w, b, y, du, uint64_t(cols), eps);                 \
  }
      TFX_LN_SMEM(1)
      TFX_LN_SMEM(2)
      TFX_LN_SMEM(3)
      TFX_LN_SMEM(4)
      TFX_LN_SMEM(6)
      TFX_LN_SMEM(8)
#undef TFX_LN_SMEM
    }
  }
  if (vec && dv <= 32 * 16) {
    TFX_REQUIRE(cols / 8 < (int64_t(1) << 31), op, "cols", "too many columns for one call");
    const unsigned grid = unsigned((cols + 7) / 8);
    const uint32_t du = uint32_t(d);
#define TFX_LN_WARP(NVV)                                                                \
  if (dv <= 32 * NVV) {                                                                   \
    return bias ? launch_kernel(op, ln_warp_kernel<T, NVV, true>, dim3(grid), dim3(256), 0,     \
                                stream, 1, x, w, b, y, du, uint64_t(cols), eps)                  \
                : launch_kernel(op, ln_warp_kernel<T, NVV, false>, dim3(grid), dim3(256), 0,    \
                                stream, 1, x, w, b, y, du, uint64_t(cols), eps);                 \
  }
    TFX_LN_WARP(1)
    TFX_LN_WARP(2)
    TFX_LN_WARP(3)
    TFX_LN_WARP(4)
    TFX_LN_WARP(6)
    TFX_LN_WARP(8)
    TFX_LN_WARP(12)
    TFX_LN_WARP(16)
#undef TFX_LN_WARP
  }
  TFX_REQUIRE(cols < (int64_t(1) << 31), op, "cols", "too many columns for one call");
  if (vec && dv <= 256 * 8) {
    const unsigned grid = unsigned(cols);
    const uint32_t du = uint32_t(d);
#define TFX_LN_CTA(NVV)                                                                   \
  if (dv <= 256 * NVV) {                                                                   \
    return bias ? launch_kernel(op, ln_cta_kernel<T, NVV, true>, dim3(grid), dim3(256), 0,  \
                                stream, 1, x, w, b, y, du, eps)                             \
                : launch_kernel(op, ln_cta_kernel<T, NVV, false>, dim3(grid), dim3(256), 0, \
                                stream, 1, x, w, b, y, du, eps);                            \
  }
    TFX_LN_CTA(2)
    TFX_LN_CTA(4)
    TFX_LN_CTA(8)
#undef TFX_LN_CTA
  }
  return launch_kernel(op, ln_generic_kernel<T>, dim3(unsigned(cols)), dim3(256), 0, stream, 1, x,
                       w, b, y, uint64_t(d), eps);
}

// ---- RMSNorm feature-last: cluster-split register tiles ---------------------------

template <typename T, int VEC>
struct RowVec {
  T v[VEC];
};

template <typename T, int VEC>
__device__ __forceinline__ RowVec<T, VEC> load_rows(const T* p) {
  RowVec<T, VEC> r;
  if constexpr (sizeof(T) * VEC == 16) {
    const V16<T> q = load16(p);
#pragma unroll
    for (int k = 0; k < VEC; ++k) r.v[k] = q.v[k];
  } else if constexpr (std::is_same_v<T, float> && VEC == 2) {
    const float2 q = ld_stream(reinterpret_cast<const float2*>(p));
    r.v[0] = q.x;
    r.v[1] = q.y;
  } else {
#pragma unroll
    for (int k = 0; k < VEC; ++k) r.v[k] = ld_stream(p + k);
  }
  return r;
}

template <typename T, int VEC>
__device__ __forceinline__ void store_rows(T* p, const RowVec<T, VEC>& r) {
  if constexpr (sizeof(T) * VEC == 16) {
    V16<T> q;
#pragma unroll
    for (int k = 0; k < VEC; ++k) q.v[k] = r.v[k];
    store16(p, q);
  } else if constexpr (std::is_same_v<T, float> && VEC == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(r.v[0], r.v[1]);
  } else {
#pragma unroll
    for (int k = 0; k < VEC; ++k) p[k] = r.v[k];
  }
}

constexpr int kRmsWarps = 8;

// One cluster of C CTAs owns tokens [tile*32*VEC, (tile+1)*32*VEC); CTA `rank`
// owns features [rank*fpc, min(width, (rank+1)*fpc)); warp w of it owns the
// features f0 + w + 8k, k < FPT; lane l owns tokens tile*32*VEC + l*VEC + [0, VEC).
template <typename T, int VEC, int FPT>
__global__ void __launch_bounds__(kRmsWarps * 32) rms_cluster_kernel(
    const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, uint32_t rows,
    uint32_t width, uint32_t fpc, T eps, T inv_width, int centered) {
  pdl_enter();
  constexpr int TR = 32 * VEC;  // tokens per tile
  __shared__ T red[kRmsWarps][TR];
  __shared__ T part[TR];
  __shared__ T scale_s[TR];
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t rank = cluster.block_rank();
  const uint32_t csize = cluster.num_blocks();
  const uint32_t tile = blockIdx.x / csize;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t r0 = tile * TR + lane * VEC;
  const bool row_ok = r0 < rows;  // rows % VEC == 0: a vector is all in or all out
  const uint32_t f0 = rank * fpc;
  const uint32_t f1 = min(width, f0 + fpc);

  RowVec<T, VEC> v[FPT];
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + kRmsWarps * k;
    if (row_ok && f < f1) v[k] = load_rows<T, VEC>(x + uint64_t(f) * rows + r0);
  }
  T ss[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) ss[j] = T(0);
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + kRmsWarps * k;
    if (row_ok && f < f1)
#pragma unroll
      for (int j = 0; j < VEC; ++j) ss[j] = add_rn(ss[j], mul_rn(v[k].v[j], v[k].v[j]));
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) red[warp][lane * VEC + j] = ss[j];
  __syncthreads();
  if (threadIdx.x < TR) {
    T s = T(0);
#pragma unroll
    for (int i = 0; i < kRmsWarps; ++i) s = add_rn(s, red[i][threadIdx.x]);
    part[threadIdx.x] = s;
  }
  cluster.sync();  // every CTA's partial sums are visible cluster-wide
  if (threadIdx.x < TR) {
    T tot = T(0);
    for (uint32_t c = 0; c < csize; ++c) tot = add_rn(tot, *cluster.map_shared_rank(&part[threadIdx.x], c));
    // scale = 1 / sqrt(mean_sq * (1/width) + eps)  (cpu-kernels lib.rs:571)
    scale_s[threadIdx.x] = div_rn(T(1), sqrt_rn(add_rn(mul_rn(tot, inv_width), eps)));
  }
  cluster.sync();  // no CTA leaves while a peer may still read its partials
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + kRmsWarps * k;
    if (row_ok && f < f1) {
      const T wf = __ldg(w + f);
      const T wt = centered ? add_rn(T(1), wf) : wf;
      RowVec<T, VEC> o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) o.v[j] = mul_rn(mul_rn(v[k].v[j], scale_s[lane * VEC + j]), wt);
      store_rows<T, VEC>(y + uint64_t(f) * rows + r0, o);
    }
  }
}

// Any width / alignment: a CTA per 32-token tile, two passes over the features
// (the second read mostly hits L2).
template <typename T>
__global__ void __launch_bounds__(256) rms_generic_kernel(const T* x, const T* __restrict__ w,
                                                          T* y, uint64_t rows,
                                                          uint64_t width, T eps, T inv_width,
                                                          int centered) {
  pdl_enter();
  __shared__ T red[8][32];
  __shared__ T scale_s[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint64_t r = uint64_t(blockIdx.x) * 32 + lane;
  T ss = T(0);
  if (r < rows)
    for (uint64_t f = warp; f < width; f += 8) {
      const T v = x[f * rows + r];
      ss = add_rn(ss, mul_rn(v, v));
    }
  red[warp][lane] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    T s = T(0);
    for (int i = 0; i < 8; ++i) s = add_rn(s, red[i][threadIdx.x]);
    scale_s[threadIdx.x] = div_rn(T(1), sqrt_rn(add_rn(mul_rn(s, inv_width), eps)));
  }
  __syncthreads();
  if (r < rows)
    for (uint64_t f = warp; f < width; f += 8) {
      const T wt = centered ? add_rn(T(1), w[f]) : w[f];
      y[f * rows + r] = mul_rn(mul_rn(x[f * rows + r], scale_s[lane]), wt);
    }
}

// Cluster-free alternative for f32: a CTA per 32-token tile; pass 1 streams
// the tile's features (U loads in flight per thread) into per-token sums of
// squares, pass 2 re-reads the tile -- from L2, which holds it since pass 1 --
// and writes the scaled values.
template <int U>
__global__ void __launch_bounds__(256) rms_tile_kernel(const float* x,
                                                       const float* __restrict__ w, float* y,
                                                       uint32_t rows, uint32_t width, float eps,
                                                       float inv_width, int centered) {
  pdl_enter();
  __shared__ float red[8][32];
  __shared__ float scale_s[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t r = blockIdx.x * 32 + lane;
  const bool ok = r < rows;
  float ss = 0.0f;
  for (uint32_t f0 = warp; f0 < width; f0 += 8 * U) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t f = f0 + 8 * u;
      v[u] = (ok && f < width) ? ld_stream(x + uint64_t(f) * rows + r) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) ss = __fadd_rn(ss, __fmul_rn(v[u], v[u]));
  }
  red[warp][lane] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = __fadd_rn(s, red[i][threadIdx.x]);
    scale_s[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, inv_width), eps)));
  }
  __syncthreads();
  const float sc = scale_s[lane];
  for (uint32_t f0 = warp; f0 < width; f0 += 8 * U) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t f = f0 + 8 * u;
      v[u] = (ok && f < width) ? __ldcg(x + uint64_t(f) * rows + r) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t f = f0 + 8 * u;
      if (ok && f < width) {
        const float wf = __ldg(w + f);
        const float wt = centered ? __fadd_rn(1.0f, wf) : wf;
        y[uint64_t(f) * rows + r] = __fmul_rn(__fmul_rn(v[u], sc), wt);
      }
    }
  }
}

// Split variant, pass A: CTA (tile, chunk) reduces tokens [tile*32*VEC, +32*VEC)
// over features [chunk*fpc, +fpc) (warp w owns features f0 + w + 8k) and writes
// one partial sum of squares per token to partial[chunk * rows + token].
template <int VEC, int FPT>
__global__ void __launch_bounds__(256) rms_partial_kernel(const float* __restrict__ x,
                                                          float* __restrict__ partial,
                                                          uint32_t rows, uint32_t width,
                                                          uint32_t fpc) {
  pdl_enter();
  constexpr int TR = 32 * VEC;
  __shared__ float red[8][TR];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t r0 = blockIdx.x * TR + lane * VEC;
  const bool row_ok = r0 < rows;
  const uint32_t f0 = blockIdx.y * fpc;
  const uint32_t f1 = min(width, f0 + fpc);
  RowVec<float, VEC> v[FPT];
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + 8 * k;
    if (row_ok && f < f1) v[k] = load_rows<float, VEC>(x + uint64_t(f) * rows + r0);
  }
  float ss[VEC];
#pragma unroll
  for (int j = 0; j < VEC; ++j) ss[j] = 0.0f;
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + 8 * k;
    if (row_ok && f < f1)
#pragma unroll
      for (int j = 0; j < VEC; ++j) ss[j] = __fadd_rn(ss[j], __fmul_rn(v[k].v[j], v[k].v[j]));
  }
#pragma unroll
  for (int j = 0; j < VEC; ++j) red[warp][lane * VEC + j] = ss[j];
  __syncthreads();
  if (threadIdx.x < TR) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = __fadd_rn(s, red[i][threadIdx.x]);
    const uint32_t r = blockIdx.x * TR + threadIdx.x;
    if (r < rows) partial[uint64_t(blockIdx.y) * rows + r] = s;
  }
}

// Split variant, pass B: sums the token's partials in chunk order, then scales
// the CTA's (tile, chunk) block, re-reading x (from L2 when x fits there).
template <int VEC, int FPT>
__global__ void __launch_bounds__(256) rms_apply_kernel(const float* x,
                                                        const float* __restrict__ w,
                                                        const float* __restrict__ partial,
                                                        float* y, uint32_t rows, uint32_t width,
                                                        uint32_t fpc, uint32_t chunks, float eps,
                                                        float inv_width, int centered) {
  pdl_enter();
  constexpr int TR = 32 * VEC;
  __shared__ float scale_s[TR];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x < TR) {
    const uint32_t r = blockIdx.x * TR + threadIdx.x;
    float tot = 0.0f;
    if (r < rows)
      for (uint32_t c = 0; c < chunks; ++c) tot = __fadd_rn(tot, __ldcg(partial + uint64_t(c) * rows + r));
    scale_s[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, inv_width), eps)));
  }
  const uint32_t r0 = blockIdx.x * TR + lane * VEC;
  const bool row_ok = r0 < rows;
  const uint32_t f0 = blockIdx.y * fpc;
  const uint32_t f1 = min(width, f0 + fpc);
  RowVec<float, VEC> v[FPT];
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + 8 * k;
    if (row_ok && f < f1) v[k] = load_rows<float, VEC>(x + uint64_t(f) * rows + r0);
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < FPT; ++k) {
    const uint32_t f = f0 + warp + 8 * k;
    if (row_ok && f < f1) {
      const float wf = __ldg(w + f);
      const float wt = centered ? __fadd_rn(1.0f, wf) : wf;
      RowVec<float, VEC> o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) o.v[j] = __fmul_rn(__fmul_rn(v[k].v[j], scale_s[lane * VEC + j]), wt);
      store_rows<float, VEC>(y + uint64_t(f) * rows + r0, o);
    }
  }
}

// Kernel choice for the f32 feature-last RMSNorm: 0 = automatic, 1 = cluster,
// 2 = tile, 3 = split, 4 = 16-CTA cluster, 5 = TMA-pipelined stream, 6 = TMA
// box ring into registers, 7 = the ring on 32-token tiles shared by a CTA
// pair; TFX_RMS_KERNEL overrides it for tuning runs.
int rms_kernel_choice() {
  static const int choice = [] {
    const char* e = getenv("TFX_RMS_KERNEL");
    if (!e) return 0;
    const std::string s(e);
    return s == "cluster" ? 1
           : s == "tile"    ? 2
           : s == "split"   ? 3
           : s == "cluster16" ? 4
           : s == "stream"  ? 5
           : s == "ring"    ? 6
           : s == "pair"    ? 7
                            : 0;
  }();
  return choice;
}

template <typename T, int VEC, int FPT>
cudaError_t launch_rms_cluster(const T* x, const T* w, T* y, uint32_t rows, uint32_t width,
                               int csize, uint32_t fpc, T eps, T inv_width, int centered,
                               cudaStream_t stream) {
  const uint32_t tiles = (rows + 32 * VEC - 1) / (32 * VEC);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * csize, 1, 1);
  cfg.blockDim = dim3(kRmsWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (csize > 8) {
    const cudaError_t err = cudaFuncSetAttribute(
        rms_cluster_kernel<T, VEC, FPT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err != cudaSuccess) return err;
  }
  return cudaLaunchKernelEx(&cfg, rms_cluster_kernel<T, VEC, FPT>, x, w, y, rows, width, fpc, eps,
                            inv_width, centered);
}

// Split variant: pass A (partials) and pass B (scale + write) over a grid of
// (token tiles, 64-feature chunks). The partial sums live in a stream-ordered
// scratch allocation of chunks * rows floats, released on the same stream.
// Returns 1 (nothing launched) when the scratch cannot be had.
int rms_split(const char* op, const float* x, const float* w, float* y, uint32_t rows,
              uint32_t width, int vec, int centered, float eps, float inv_width,
              cudaStream_t stream) {
  constexpr int FPT = 8;
  const uint32_t fpc = 8 * FPT;
  const uint32_t chunks = (width + fpc - 1) / fpc;
  const uint32_t tr = 32 * uint32_t(vec);
  const uint32_t tiles = (rows + tr - 1) / tr;
  if (chunks > 65535) return 1;
  float* partial = nullptr;
  if (scratch_malloc(reinterpret_cast<void**>(&partial), size_t(chunks) * rows * 4, stream) !=
      cudaSuccess) {
    cudaGetLastError();  // clear the allocation failure; the caller falls back
    return 1;
  }
  const dim3 grid(tiles, chunks);
  auto run = [&](auto partial_k, auto apply_k) {
    int rc = launch_kernel(op, partial_k, grid, dim3(256), 0, stream, 1, x, partial, rows, width,
                           fpc);
    if (rc == TFX_OK)
      rc = launch_kernel(op, apply_k, grid, dim3(256), 0, stream, 1, x, w,
                         static_cast<const float*>(partial), y, rows, width, fpc, chunks, eps,
                         inv_width, centered);
    return rc;
  };
  int rc;
  if (vec == 4) rc = run(rms_partial_kernel<4, FPT>, rms_apply_kernel<4, FPT>);
  else if (vec == 2) rc = run(rms_partial_kernel<2, FPT>, rms_apply_kernel<2, FPT>);
  else rc = run(rms_partial_kernel<1, FPT>, rms_apply_kernel<1, FPT>);
  cudaFreeAsync(partial, stream);
  return rc;
}

// Picks the kernel and its (VEC, FPT, cluster size) for the shape; the generic
// kernel runs when nothing else covers it.
template <typename T>
int rmsnorm_last(const char* op, const T* x, const T* w, T* y, int64_t rows, int64_t width,
                 int centered, T eps, cudaStream_t stream) {
  clear_error();
  TFX_REQUIRE(rows >= 0 && width >= 0, op, "shape", "extents must be non-negative");
  if (rows == 0 || width == 0) return TFX_OK;
  TFX_REQUIRE(x, op, "x", "null pointer");
  TFX_REQUIRE(w, op, "weight", "null pointer");
  TFX_REQUIRE(y, op, "y", "null pointer");
  const size_t bytes = size_t(rows) * size_t(width) * sizeof(T);
  TFX_REQUIRE(y == x || !overlaps(x, bytes, y, bytes), op, "y", "partially overlaps x");
  TFX_REQUIRE(!overlaps(w, size_t(width) * sizeof(T), y, bytes), op, "weight", "overlaps y");
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  // f32: 1/width as the f32 reciprocal (lib.rs:560); f64: 1.0 / width.
  const T inv_width = T(1) / T(width);
  const bool small = rows < (int64_t(1) << 31) && width < (int64_t(1) << 31) &&
                     uint64_t(rows) * uint64_t(width) < (uint64_t(1) << 40);
  int vec = 1;
  constexpr int V16N = 16 / int(sizeof(T));
  if (rows % V16N == 0 && aligned(x, 16) && aligned(y, 16)) vec = V16N;
  else if (std::is_same_v<T, float> && rows % 2 == 0 && aligned(x, 8) && aligned(y, 8)) vec = 2;
  int max_cluster = 8;
  if constexpr (std::is_same_v<T, float>) {
    const int choice = rms_kernel_choice();
    if (small && choice == 2) {
      return launch_kernel(op, rms_tile_kernel<8>, dim3(unsigned((rows + 31) / 32)), dim3(256), 0,
                           stream, 1, x, w, y, uint32_t(rows), uint32_t(width), eps, inv_width,
                           centered);
    }
    // The ring kernel (TMA boxes into registers) and the streaming kernel
    // (whole tiles staged in shared memory) read x once with their loads
    // always in flight; they cover aligned shapes with rows % 4 == 0, widths
    // 513 .. 2048 and up to ~3300 respectively.
    if (small && choice == 7) {
      const int rc = rms_pair(op, x, w, y, uint32_t(rows), uint32_t(width), centered, eps,
                              inv_width, stream);
      if (rc != 1) return rc;
    }
    if (small && (choice == 0 || choice == 6)) {
      const int rc = rms_ring(op, x, w, y, uint32_t(rows), uint32_t(width), centered, eps,
                              inv_width, stream);
      if (rc != 1) return rc;
    }
    if (small && (choice == 0 || choice == 5)) {
      const int rc = rms_stream(op, x, w, y, uint32_t(rows), uint32_t(width), centered, eps,
                                inv_width, stream);
      if (rc != 1) return rc;
    }
    // The split variant re-reads x once; it wins when x stays in L2 between
    // its two passes.
    const bool fits_l2 = double(bytes) <= 0.75 * double(dev.l2_bytes);
    if (small && (choice == 3 || (choice == 0 && fits_l2)) && (rows + 127) / 128 < 65536 * 64) {
      const int rc = rms_split(op, x, w, y, uint32_t(rows), uint32_t(width), vec, centered, eps,
                               inv_width, stream);
      if (rc != 1) return rc;  // 1: scratch unavailable, take the cluster kernel
    }
    if (choice == 4) max_cluster = 16;
  }
  if (small) {
    const uint32_t r = uint32_t(rows), wd = uint32_t(width);
    // Features per CTA = 8 warps * FPT; the cluster holds up to max_cluster CTAs.
    auto try_cfg = [&](int fpt, auto launch) -> int {
      const int64_t per_cta = int64_t(kRmsWarps) * fpt;
      const int64_t csize = (width + per_cta - 1) / per_cta;
      if (csize > max_cluster) return 1;  // not covered
      const uint32_t fpc = uint32_t((width + csize - 1) / csize);
      const cudaError_t err = launch(int(csize), fpc);
      if (err != cudaSuccess)
        return fail(TFX_ERR_CUDA, op, "launch", std::string(cudaGetErrorName(err)) + ": " +
                                                     cudaGetErrorString(err));
      return TFX_OK;
    };
#define TFX_RMS_TRY(V, FPT)                                                                 \
  {                                                                                         \
    const int rc = try_cfg(FPT, [&](int cs, uint32_t fpc) {                                 \
      return launch_rms_cluster<T, V, FPT>(x, w, y, r, wd, cs, fpc, eps, inv_width, centered, \
                                           stream);                                         \
    });                                                                                     \
    if (rc != 1) return rc;                                                                 \
  }
    if constexpr (std::is_same_v<T, float>) {
      if (vec == 4) { TFX_RMS_TRY(4, 4) TFX_RMS_TRY(4, 8) TFX_RMS_TRY(4, 16) }
      else if (vec == 2) { TFX_RMS_TRY(2, 8) TFX_RMS_TRY(2, 16) TFX_RMS_TRY(2, 32) }
      else { TFX_RMS_TRY(1, 16) TFX_RMS_TRY(1, 32) TFX_RMS_TRY(1, 64) }
    } else {
      if (vec == 2) { TFX_RMS_TRY(2, 4) TFX_RMS_TRY(2, 8) TFX_RMS_TRY(2, 16) }
      else { TFX_RMS_TRY(1, 8) TFX_RMS_TRY(1, 16) TFX_RMS_TRY(1, 32) }
    }
#undef TFX_RMS_TRY
  }
  TFX_REQUIRE((rows + 31) / 32 < (int64_t(1) << 31), op, "rows", "too many rows for one call");
  return launch_kernel(op, rms_generic_kernel<T>, dim3(unsigned((rows + 31) / 32)), dim3(256), 0,
                       stream, 1, x, w, y, uint64_t(rows), uint64_t(width), eps, inv_width,
                       centered);
}

}  // namespace
}  // namespace tfx

extern "C" {

int tfx_layernorm_ff_f32(const float* x, const float* weight, const float* bias, float* y,
                         int64_t d, int64_t cols, float eps, tfx_stream_t stream) {
  return tfx::layernorm_ff<float>("tenferro-ext::layernorm_ff", x, weight, bias, y, d, cols, eps,
                                  stream);
}

int tfx_add_layernorm_ff_f32(const float* a, const float* b, const float* weight,
                             const float* bias, float* sum_out, float* y, int64_t d, int64_t cols,
                             float eps, tfx_stream_t stream) {
  using namespace tfx;
  clear_error();
  const char* op = "tenferro-ext::add_layernorm_ff";
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  TFX_REQUIRE(d >= 0 && cols >= 0, op, "shape", "extents must be non-negative");
  if (d == 0 || cols == 0) return TFX_OK;
  TFX_REQUIRE(a && b && weight && y, op, a ? (b ? (weight ? "y" : "weight") : "b") : "a",
              "null pointer");
  const size_t bytes = size_t(d) * size_t(cols) * 4;
  auto ok_alias = [&](const void* p, const void* q) { return p == q || !overlaps(p, bytes, q, bytes); };
  TFX_REQUIRE(ok_alias(a, y) && ok_alias(b, y), op, "y", "partially overlaps an input");
  TFX_REQUIRE(!sum_out || (ok_alias(a, sum_out) && ok_alias(b, sum_out) &&
                           !overlaps(sum_out, bytes, y, bytes)),
              op, "sum_out", "overlaps y or partially overlaps an input");
  TFX_REQUIRE(!overlaps(weight, size_t(d) * 4, y, bytes) &&
                  (!sum_out || !overlaps(weight, size_t(d) * 4, sum_out, bytes)),
              op, "weight", "overlaps an output");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  const bool vec = d % 4 == 0 && aligned(a, 16) && aligned(b, 16) && aligned(y, 16) &&
                   aligned(weight, 16) && (!bias || aligned(bias, 16)) &&
                   (!sum_out || aligned(sum_out, 16));
  const int64_t dv = d / 4;
  static const bool use_regs = [] {
    const char* e = getenv("TFX_LN_KERNEL");
    return e && std::string(e) == "regs";
  }();
  if (vec && dv <= 32 * 6 && !use_regs && cols / 8 < (int64_t(1) << 31)) {
    const unsigned grid = unsigned((cols + 7) / 8);
    const uint32_t du = uint32_t(d);
    const size_t smem = size_t(8) * 2 * size_t(d) * 4;
    float* so = sum_out ? sum_out : y;  // unused when SUM is false
#define TFX_ADD_LN(NVV, B, S)                                                                  \
  {                                                                                            \
    auto k = add_ln_smem_kernel<NVV, B, S>;                                                    \
    if (smem > 48 * 1024) {                                                                    \
      const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                                 int(smem));                                   \
      if (e != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(e));    \
    }                                                                                          \
    return launch_kernel(op, k, dim3(grid), dim3(256), smem, s, 1, a, b, weight, bias, so, y, \
                         du, uint64_t(cols), eps);                                             \
  }
#define TFX_ADD_LN_NV(NVV)                                                \
  if (dv <= 32 * NVV) {                                                   \
    if (bias) {                                                           \
      if (sum_out) TFX_ADD_LN(NVV, true, true) else TFX_ADD_LN(NVV, true, false)   \
    } else {                                                              \
      if (sum_out) TFX_ADD_LN(NVV, false, true) else TFX_ADD_LN(NVV, false, false) \
    }                                                                     \
  }
    TFX_ADD_LN_NV(1)
    TFX_ADD_LN_NV(2)
    TFX_ADD_LN_NV(3)
    TFX_ADD_LN_NV(4)
    TFX_ADD_LN_NV(6)
#undef TFX_ADD_LN_NV
#undef TFX_ADD_LN
  }
  // Other shapes: the two ops back to back (identical results by construction).
  float* tmp = sum_out;
  if (!tmp) {
    if (scratch_malloc(reinterpret_cast<void**>(&tmp), bytes, s) != cudaSuccess) {
      cudaGetLastError();
      return fail(TFX_ERR_CUDA, op, "scratch", "cannot allocate the sum");
    }
  }
  int rc = tfx_add_f32(a, b, tmp, d * cols, stream);
  if (rc == TFX_OK) rc = tfx_layernorm_ff_f32(tmp, weight, bias, y, d, cols, eps, stream);
  if (!sum_out) cudaFreeAsync(tmp, s);
  return rc;
}

int tfx_layernorm_ff_f64(const double* x, const double* weight, const double* bias, double* y,
                         int64_t d, int64_t cols, double eps, tfx_stream_t stream) {
  return tfx::layernorm_ff<double>("tenferro-infer::layer_norm", x, weight, bias, y, d, cols,
                                   eps, stream);
}

int tfx_rmsnorm_last_f32(const float* x, const float* weight, float* y, int64_t rows,
                         int64_t width, int centered, float eps, tfx_stream_t stream) {
  return tfx::rmsnorm_last<float>("tenferro-ext::rms_norm_last", x, weight, y, rows, width,
                                  centered ? 1 : 0, eps, stream);
}

int tfx_rmsnorm_last_f64(const double* x, const double* weight, double* y, int64_t rows,
                         int64_t width, int centered, double eps, tfx_stream_t stream) {
  return tfx::rmsnorm_last<double>("tenferro-infer::rms_norm", x, weight, y, rows, width,
                                   centered ? 1 : 0, eps, stream);
}

}  // extern "C"

// ---- RMSNorm without any allocation ------------------------------------------------
//
// tfx_rmsnorm_last_f32 takes the split kernels' partial sums from a
// stream-ordered allocation. Some callers cannot let a library allocate device
// memory at call time: a serving process whose HBM is reserved up front by its
// own allocator (a cudaMallocAsync there can fail or fragment the pool), or a
// latency-critical loop that must not take the allocator's locks, grow a pool
// or risk the implicit synchronisation of an allocation. For them this entry
// point runs the same two kernels on a fixed scratch array that is part of the
// library's device image: it is reserved on every GPU that loads libtfx, for as
// long as the process lives, and no call allocates or frees anything.

// Partial sums of squares of the split kernels: (width / 64 rounded up) * rows
// floats per call, at most 2^20 (4 MiB).
constexpr size_t kStaticScratchFloats = size_t(1) << 20;
static __device__ __align__(256) float g_rms_static_scratch[kStaticScratchFloats];

namespace tfx {
namespace {

// Device address of g_rms_static_scratch on the current device. Host code only
// sees a host-side stand-in for the array, so the address is looked up with
// cudaGetSymbolAddress once per device (with that device current) and cached.
float* static_scratch(const char* op, int* status) {
  constexpr int kMaxDev = 64;
  static std::once_flag once[kMaxDev];
  static float* addr[kMaxDev];
  static cudaError_t err[kMaxDev];
  int dev = -1;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    *status = fail(TFX_ERR_CUDA, op, "scratch", "cannot read the current device");
    return nullptr;
  }
  std::call_once(once[dev], [dev] {
    err[dev] = cudaGetSymbolAddress(reinterpret_cast<void**>(&addr[dev]), g_rms_static_scratch);
  });
  if (err[dev] != cudaSuccess || addr[dev] == nullptr) {
    *status = fail(TFX_ERR_CUDA, op, "scratch",
                   std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(err[dev]));
    return nullptr;
  }
  *status = TFX_OK;
  return addr[dev];
}

}  // namespace
}  // namespace tfx

extern "C" int tfx_rmsnorm_last_f32_noalloc(const float* x, const float* weight, float* y,
                                            int64_t rows, int64_t width, int centered,
                                            float eps, tfx_stream_t stream) {
  using namespace tfx;
  clear_error();
  const char* op = "tenferro-ext::rms_norm_last";
  TFX_REQUIRE(rows >= 0 && width >= 0, op, "shape", "extents must be non-negative");
  if (rows == 0 || width == 0) return TFX_OK;
  TFX_REQUIRE(x, op, "x", "null pointer");
  TFX_REQUIRE(weight, op, "weight", "null pointer");
  TFX_REQUIRE(y, op, "y", "null pointer");
  const size_t bytes = size_t(rows) * size_t(width) * 4;
  TFX_REQUIRE(y == x || !overlaps(x, bytes, y, bytes), op, "y", "partially overlaps x");
  TFX_REQUIRE(!overlaps(weight, size_t(width) * 4, y, bytes), op, "weight", "overlaps y");
  const int64_t chunks = (width + 63) / 64;
  if (rows >= (int64_t(1) << 31) || chunks > 65535 ||
      uint64_t(chunks) * uint64_t(rows) > kStaticScratchFloats)
    return fail(TFX_ERR_UNSUPPORTED, op, "shape",
                "rows x ceil(width/64) = " + std::to_string(chunks) + " x " +
                    std::to_string(rows) + " partial sums exceed the fixed scratch of " +
                    std::to_string(kStaticScratchFloats) +
                    " floats; split the rows over several calls or use tfx_rmsnorm_last_f32");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  float* partial = static_scratch(op, &st);
  if (st != TFX_OK) return st;
  int vec = 1;
  if (rows % 4 == 0 && aligned(x, 16) && aligned(y, 16)) vec = 4;
  else if (rows % 2 == 0 && aligned(x, 8) && aligned(y, 8)) vec = 2;
  // Pass A writes every partial that pass B reads, so nothing in the scratch
  // needs clearing between calls.
  constexpr int FPT = 8;
  const uint32_t r = uint32_t(rows), wd = uint32_t(width);
  const uint32_t fpc = 8 * FPT, nch = uint32_t(chunks);
  const float inv_width = 1.0f / float(width);
  const dim3 grid((r + 32 * vec - 1) / (32 * vec), nch);
  if (vec == 4) {
    rms_partial_kernel<4, FPT><<<grid, 256, 0, stream>>>(x, partial, r, wd, fpc);
    rms_apply_kernel<4, FPT><<<grid, 256, 0, stream>>>(x, weight, partial, y, r, wd, fpc, nch,
                                                       eps, inv_width, centered ? 1 : 0);
  } else if (vec == 2) {
    rms_partial_kernel<2, FPT><<<grid, 256, 0, stream>>>(x, partial, r, wd, fpc);
    rms_apply_kernel<2, FPT><<<grid, 256, 0, stream>>>(x, weight, partial, y, r, wd, fpc, nch,
                                                       eps, inv_width, centered ? 1 : 0);
  } else {
    rms_partial_kernel<1, FPT><<<grid, 256, 0, stream>>>(x, partial, r, wd, fpc);
    rms_apply_kernel<1, FPT><<<grid, 256, 0, stream>>>(x, weight, partial, y, r, wd, fpc, nch,
                                                       eps, inv_width, centered ? 1 : 0);
  }
  return check_launch(op);
}
