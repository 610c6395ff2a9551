// gemm_epilogue.cu -- the GEMM-epilogue fusions of the MLP projection:
// GemmGegluOp (crates/tenferro-ext/src/gemm_geglu.rs:114-240, the projection
// then geglu_into) and GemmBiasOp with an activation (gemm_bias.rs:76-142; on
// CUDA the reference runs a GEMM, then FusedScope::bias_act_first,
// cuda_fused.rs:704, kernel fused_bias_act, fused.cu:137), as one tcgen05
// kernel whose epilogue reads the accumulators from tensor memory.
//
// Layouts (the reference's column-major ones): x is feature-first
// (in_dim, length), element (i, t) at i + in_dim*t; weight is (in_dim, out)
// with element (i, o) at i + in_dim*o; the projection is
//   p[o, t] = bias[o] + sum_i x[i, t] * weight[i, o]
// (cpu-kernels lib.rs:274-288, input_mul_weight_transpose_bias_into), and
//   GeGLU:    y[j + I*t] = gelu_erf(p[j, t]) * p[I + j, t]   (out = 2I, lib.rs:516-538)
//   bias+act: y[o + out*t] = act(p[o, t])
// Only y is written: the (out, length) projection never reaches HBM.
//
// Arithmetic. f32 accuracy on the tensor cores by the 3xTF32 split: every
// operand value v = hi + lo with hi and lo tf32 roundings (cvt.rna), and
// x.w ~ xh.wh + xh.wl + xl.wh (the dropped xl.wl is ~2^-22 relative), f32
// accumulation in TMEM. A prep kernel writes hi and lo of x and of the weight
// into a stream-ordered scratch, with K padded to a multiple of 32 with zeros,
// so every tensor-map constraint holds whatever the caller's shapes and
// alignment. The epilogue adds the bias (one rounding) and applies the
// reference's exact-erf GELU (tfx_math.h, bit-identical to gelu_erf_f32) or
// ReLU. The result differs from the reference's f32 GEMM by summation order
// and the split (f32 tolerance), not by the epilogue arithmetic.
//
// Non-finite operands (and |v| >= 2^60, whose split could overflow) take an
// exact path: the prep kernel flags every 128-token tile of x that holds one
// (and the whole call when the weight does); the tensor-core kernel skips
// those tiles and a SIMT kernel computes them with the reference's operation
// order (sequential sum from the bias, each product rounded, no FMA), so
// inf / NaN propagate as in the reference.
//
// Kernel (one persistent CTA per SM, 320 threads):
//   warp 0  TMA producer: per K chunk of 32, the x tile (128 tokens) hi and lo
//           and the weight tile (256 output rows) hi and lo, 96 KB, into one
//           of two shared-memory stages (128-byte swizzled, K-major);
//   warp 1  TMEM owner and MMA issuer: 12 tcgen05.mma.kind::tf32 (M 128,
//           N 256, K 8) per chunk into one of two 256-column partials;
//   warps 2-9 epilogue: two warps per TMEM lane quarter (one token per
//           thread, 128 of the 256 columns per warp) add every chunk's
//           partial into f32 registers and release it to the MMA warp, then
//           at the tile's end apply bias, GeGLU / activation and store.
// For GeGLU the 256 columns are projection rows [n0, n0 + 128) (the GELU'd
// half) and [I + n0, I + n0 + 128) (the gate half), so a thread holding
// column c also holds column 128 + c. Every mbarrier wait is
// bounded (~1 s); a role that gives up counts it, sets a CTA-wide abort flag
// that ends the other roles' waits, and the CTA drains its own copies and
// MMAs (bounded) and frees its TMEM before it exits.

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "causal_tiles.cuh"
#include "common.cuh"
#include "internal.h"
#include "tc.cuh"
#include "tfx_math.h"
#include "tma.cuh"

// Bounded waits of the GEMM-epilogue kernel that gave up, per device.
static __device__ uint32_t g_gemm_wait_timeouts;

namespace tfx {
namespace {

constexpr int kEpiGeglu = 0;
constexpr int kEpiBiasAct = 1;

constexpr int kGThreads = 320;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kBM = 128;  // tokens per tile
constexpr int kBN = 256;  // projection rows per tile
constexpr int kBK = 32;   // K padding of the scratch operands, and the largest stage
constexpr int kMaxStages = 4;
// Shared memory: the stage ring holds 192 KB whatever the stage width (two
// stages of K 32, or four of K 16), plus alignment slack.
constexpr size_t kGemmSmem = size_t(2) * (2 * kBM + 2 * kBN) * kBK * 4 + 1024;
// + a 32 x 32 staging tile per epilogue warp (stage_rows)
constexpr size_t kGemmStage = size_t(kEpiWarps) * 32 * 32 * 4;
constexpr size_t kGemmSmemAll = kGemmSmem + kGemmStage;
constexpr long long kGemmWait = 1LL << 31;  // ~1 s at B200 clocks
constexpr float kSplitLimit = 1152921504606846976.0f;  // 2^60

struct GemmArgs {
  float* y;
  const float* bias;
  const uint32_t* flags;  // [mtiles] x tiles with a non-finite value, then [1] the weight
  uint32_t length;        // tokens
  uint32_t nk;            // K chunks of 32
  uint32_t nout;          // outputs per token: I (GeGLU) or out_dim (bias + act)
  uint32_t inter;         // GeGLU: I, the row offset of the gate half
  uint32_t mtiles, ntiles;
  int vec4;               // every output row 16-byte aligned and nout % 4 == 0
  // batched weights (bias + act only): tokens [b * batch_tokens, (b + 1) *
  // batch_tokens) use weight rows [b * batch_wrows, ...); 0 = one weight
  uint32_t batch_tokens, batch_wrows;
  // causal batches (batched, batch_tokens == nout or == in_dim; t_b = the
  // token's index in its batch): kCausalOut: only outputs o <= t_b are wanted
  // (only the live tiles are computed, the others left unwritten); kCausalK:
  // x[t][i] = 0 for i > t_b (a tile contracts up to its last token; the
  // chunks are split evenly over the CTAs, piece p of a tile writes slot p,
  // y + p * slot_stride).
  uint32_t causal;
  uint32_t mb;         // 128-token tiles per batch (causal modes)
  uint64_t items;      // tiles (kCausalOut: live tiles) dealt round robin
  uint64_t slot_stride;
  CausalKSplit split;  // kCausalK
  // batched only: y of batch b is (nout, batch_tokens), token-contiguous:
  // y[b * nout * batch_tokens + o * batch_tokens + t_b]
  int out_t;
  // the call runs on CTA pairs (gemm_pair_tc_kernel): items and the causal
  // schedules count 256-token pair rows
  int pair;
  // identity epilogue into row-major y: each warp's 32 token rows go out
  // through a shared-memory tile, 32 consecutive outputs of one row per store
  int stage_rows;
};

// A run of K stages [s0, s1) of tile (m, n) that one CTA computes, written
// to output slot `slot`.
struct GemmPiece {
  uint32_t m, n, s0, s1, slot;
  bool skip;  // a tile with a non-finite operand (the SIMT kernel's)
};

constexpr uint32_t kCausalOut = 1;
constexpr uint32_t kCausalK = 2;

// First weight row of the batch that token t belongs to.
__device__ __forceinline__ uint32_t batch_wrow(const GemmArgs& a, uint32_t t) {
  return a.batch_tokens ? (t / a.batch_tokens) * a.batch_wrows : 0u;
}

__device__ __forceinline__ float tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return __uint_as_float(r);
}

// ---- prep: hi / lo split with K padding ---------------------------------------------
//
// src (in_dim, cols) -> hi, lo (kp, cols_pad), element (k, c) at k + kp*c,
// zero for k >= in_dim or c >= cols (the padding keeps every TMA box of the
// kernel inside its tensor). A column holding a value that cannot be split
// safely (not finite, or |v| >= 2^60) sets flags[c >> shift].
template <int VEC>
__global__ void __launch_bounds__(256) split_pad_kernel(const float* __restrict__ src,
                                                        uint32_t in_dim, uint32_t cols,
                                                        uint32_t cols_pad, uint32_t kp,
                                                        float* __restrict__ hi,
                                                        float* __restrict__ lo,
                                                        uint32_t* __restrict__ flags,
                                                        uint32_t shift) {
  pdl_enter();
  const uint32_t kq = kp / 4;  // float4 groups per padded column
  const uint64_t total = uint64_t(kq) * cols_pad;
  for (uint64_t g = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t c = uint32_t(g / kq), k0 = uint32_t(g % kq) * 4;
    const float* s = src + uint64_t(c) * in_dim;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (c >= cols) {
      // padding column: zeros
    } else if (VEC == 4 && k0 + 4 <= in_dim) {
      const float4 q = ld_stream(reinterpret_cast<const float4*>(s + k0));
      v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = k0 + j < in_dim ? ld_stream(s + k0 + j) : 0.0f;
    }
    float h[4], l[4];
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!(fabsf(v[j]) < kSplitLimit)) {  // inf, NaN, huge: the SIMT path computes the tile
        bad = true;
        h[j] = 0.0f;
        l[j] = 0.0f;
      } else {
        h[j] = tf32_rna(v[j]);
        l[j] = tf32_rna(__fsub_rn(v[j], h[j]));  // v - h is exact
      }
    }
    const uint64_t o = uint64_t(c) * kp + k0;
    *reinterpret_cast<float4*>(hi + o) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + o) = make_float4(l[0], l[1], l[2], l[3]);
    if (bad) flags[c >> shift] = 1u;
  }
}

// ---- the tensor-core kernel ----------------------------------------------------------

struct GemmShared {
  // smem stages: TMA -> MMA (full) and MMA -> TMA (empty); TMEM partial
  // buffers: MMA -> epilogue (part_full) and epilogue -> MMA (part_empty)
  uint64_t full[kMaxStages], empty[kMaxStages], part_full[2], part_empty[2], drain;
  uint32_t tmem_base;
  int abort;
};

// Bounded wait on `bar` for the phase of the given parity; also ends when
// another role of the CTA has given up. Returns false when it did not
// complete (the first role to give up counts it and raises the abort flag).
__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity, GemmShared* sh) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(&sh->abort)) return false;
    if (clock64() - t0 > kGemmWait) {
      if (atomicExch(&sh->abort, 1) == 0) atomicAdd(&g_gemm_wait_timeouts, 1u);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool tile_skipped(const GemmArgs& a, uint32_t m) {
  return __ldcg(a.flags + m) != 0u || __ldcg(a.flags + a.mtiles) != 0u;
}

// The CTA's first work item.
__device__ __forceinline__ uint64_t first_item(const GemmArgs& a) {
  return a.causal == kCausalK ? a.split.start(blockIdx.x) : uint64_t(blockIdx.x);
}

// The CTA's next piece of work from item i (advanced past it); false at the
// end. Every role of the CTA walks the same sequence.
template <int SK>
__device__ __forceinline__ bool next_piece(const GemmArgs& a, uint32_t nst, uint64_t& i,
                                           GemmPiece& p) {
  if (a.causal == kCausalK) {
    // 128-key chunks: kBM / SK stages each
    const uint64_t end = a.split.start(blockIdx.x + 1);
    if (i >= end) return false;
    const uint32_t batch = uint32_t(i / a.split.per_batch);
    const uint64_t r = i - uint64_t(batch) * a.split.per_batch;
    const uint32_t lm = CausalKSplit::row_of(r);
    const uint32_t c0 = uint32_t(r - CausalKSplit::prefix(lm));
    const uint32_t c1 = uint32_t(min(uint64_t(lm) + 1, uint64_t(c0) + (end - i)));
    p.m = batch * a.mb + lm;
    p.n = 0;
    p.s0 = c0 * (kBM / SK);
    p.s1 = min(nst, c1 * (kBM / SK));
    p.slot = blockIdx.x - a.split.owner(a.split.first(batch, lm));
    p.skip = tile_skipped(a, p.m);
    i += c1 - c0;
    return true;
  }
  for (; i < a.items; i += gridDim.x) {
    if (a.causal == kCausalOut) {
      const uint64_t per = live_prefix(a.mb);
      const uint32_t batch = uint32_t(i / per);
      const uint64_t r = i - uint64_t(batch) * per;
      const uint32_t lm = live_row(r);
      p.m = batch * a.mb + lm;
      p.n = uint32_t(r - live_prefix(lm));
    } else {
      p.m = uint32_t(i / a.ntiles);
      p.n = uint32_t(i - uint64_t(p.m) * a.ntiles);
    }
    if (tile_skipped(a, p.m)) continue;
    p.s0 = 0;
    p.s1 = nst;
    p.slot = 0;
    p.skip = false;
    i += gridDim.x;
    return true;
  }
  return false;
}

template <int EPI, int ACT>
__device__ __forceinline__ float epi_act(float v) {
  if constexpr (EPI == kEpiBiasAct && ACT == TFX_ACT_GELU_ERF) return math::gelu_mlx(v);
  else if constexpr (EPI == kEpiBiasAct && ACT == TFX_ACT_RELU) return v > 0.0f ? v : 0.0f;
  else return v;
}

// The epilogue of one thread: token t's 128 sums in acc for output tile n,
// column half `half` (GeGLU: 64 values and their 64 gates), with bias,
// activation or GeGLU, stored into output slot `slot` (split contractions).
template <int EPI, int ACT, bool BIAS>
__device__ __forceinline__ void epi_store(const GemmArgs& a, uint32_t t, uint32_t n, uint32_t half,
                                          uint32_t slot, float* acc) {
  if constexpr (EPI == kEpiGeglu) {
    const uint32_t j0 = n * (kBN / 2) + 64 * half;  // first output row of this thread
    if (j0 >= a.nout) return;
    const uint32_t valid = min(64u, a.nout - j0);
    if constexpr (BIAS) {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (uint32_t(j) < valid) {
          acc[j] = __fadd_rn(acc[j], __ldg(a.bias + j0 + j));
          acc[64 + j] = __fadd_rn(acc[64 + j], __ldg(a.bias + a.inter + j0 + j));
        }
    }
    float* yr = a.y + uint64_t(t) * a.nout + j0;
#pragma unroll
    for (int c = 0; c < 64; c += 4) {
      const float2 g0 = math::gelu_mlx2(make_float2(acc[c], acc[c + 1]));
      const float2 g1 = math::gelu_mlx2(make_float2(acc[c + 2], acc[c + 3]));
      const float4 o = make_float4(__fmul_rn(g0.x, acc[64 + c]), __fmul_rn(g0.y, acc[65 + c]),
                                   __fmul_rn(g1.x, acc[66 + c]), __fmul_rn(g1.y, acc[67 + c]));
      if (a.vec4 && uint32_t(c) + 4 <= valid) {
        *reinterpret_cast<float4*>(yr + c) = o;
      } else {
        if (uint32_t(c) < valid) yr[c] = o.x;
        if (uint32_t(c) + 1 < valid) yr[c + 1] = o.y;
        if (uint32_t(c) + 2 < valid) yr[c + 2] = o.z;
        if (uint32_t(c) + 3 < valid) yr[c + 3] = o.w;
      }
    }
  } else {
    const uint32_t o0 = n * kBN + 128 * half;  // first output row of this thread
    if (o0 >= a.nout) return;
    const uint32_t valid = min(128u, a.nout - o0);
    if (a.out_t) {  // identity epilogue; a warp stores 32 consecutive tokens
      const uint32_t b = t / a.batch_tokens, tb = t - b * a.batch_tokens;
      float* yc = a.y + uint64_t(slot) * a.slot_stride +
                  (uint64_t(b) * a.nout + o0) * a.batch_tokens + tb;
#pragma unroll
      for (int c = 0; c < 128; ++c)  // fully unrolled: acc stays in registers
        if (uint32_t(c) < valid) yc[uint64_t(c) * a.batch_tokens] = acc[c];
      return;
    }
    float* yr = a.y + uint64_t(slot) * a.slot_stride + uint64_t(t) * a.nout + o0;
#pragma unroll
    for (int c = 0; c < 128; c += 4) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = acc[c + j];
        if constexpr (BIAS)
          if (uint32_t(c + j) < valid) v[j] = __fadd_rn(v[j], __ldg(a.bias + o0 + c + j));
      }
      if constexpr (ACT == TFX_ACT_GELU_ERF) {
        const float2 g0 = math::gelu_mlx2(make_float2(v[0], v[1]));
        const float2 g1 = math::gelu_mlx2(make_float2(v[2], v[3]));
        v[0] = g0.x; v[1] = g0.y; v[2] = g1.x; v[3] = g1.y;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = epi_act<EPI, ACT>(v[j]);
      }
      if (a.vec4 && uint32_t(c) + 4 <= valid) {
        *reinterpret_cast<float4*>(yr + c) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (uint32_t(c + j) < valid) yr[c + j] = v[j];
      }
    }
  }
}

// The identity epilogue of a warp's 32 token rows t0 .. t0 + 31 (lane = row),
// 128 outputs each from o0, into row-major y: staged through the warp's 32 x
// 32 shared tile (element (row r, column j) at r * 32 + (j ^ r): no bank
// conflicts either way) so that every store writes 32 consecutive outputs of
// one row, instead of 32 rows' 16 bytes each.
__device__ __forceinline__ void epi_store_staged(const GemmArgs& a, uint32_t t0, uint32_t lane,
                                                 uint32_t o0, uint32_t slot, const float* acc,
                                                 float* stage) {
  const uint32_t valid = min(128u, a.nout - o0);
  float* yb = a.y + uint64_t(slot) * a.slot_stride + uint64_t(t0) * a.nout + o0;
#pragma unroll
  for (int c = 0; c < 128; c += 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) stage[lane * 32 + (uint32_t(j) ^ lane)] = acc[c + j];
    __syncwarp();
    if (uint32_t(c) + lane < valid)
      for (uint32_t r = 0; r < 32; ++r)
        if (t0 + r < a.length) yb[uint64_t(r) * a.nout + c + lane] = stage[r * 32 + (lane ^ r)];
    __syncwarp();
  }
}

// Accumulation. The tensor cores' f32 accumulation is not IEEE: each MMA
// aligns the accumulator and its products to the largest exponent and keeps
// about 22 bits below it (measured: an accumulator fed all 288 MMAs of a
// 768-long contraction was off by up to 1.9e-6 of sum|x w|, ten times a
// sequential f32 sum). So every K chunk of 32 gets a fresh accumulator,
// filled in the order hi*lo, lo*hi (the small terms, accurate while the
// partial is small), then hi*hi -- 4 truncating steps at the large scale per
// chunk -- and the epilogue warps add each chunk's partial into f32 registers
// (IEEE adds), with the bias added at the end: max error 1.3e-7 of sum|x w|
// in a model of the hardware calibrated on the measurement above, on a par
// with the sequential f32 sum of the reference (1.6e-7).
//
// Stages: SK K values per stage (32: 128-byte swizzled rows, two 96 KB
// stages; 16: 64-byte swizzled rows, four 48 KB stages, so a stage is freed
// and refilled after half as much MMA work). FK: K values per partial (the
// drain period). Each stage's MMAs run small products first.
template <int EPI, int ACT, bool BIAS, int SK, int FK>
__global__ void __launch_bounds__(kGThreads, 1) gemm_epi_tc_kernel(
    const __grid_constant__ CUtensorMap xh_map, const __grid_constant__ CUtensorMap xl_map,
    const __grid_constant__ CUtensorMap wh_map, const __grid_constant__ CUtensorMap wl_map,
    GemmArgs a) {
  static_assert((SK == 16 || SK == 32) && FK % SK == 0, "stage shape");
  constexpr int kStages = 2 * kBK / SK;
  constexpr uint32_t kABytes = kBM * SK * 4;
  constexpr uint32_t kBBytes = kBN * SK * 4;
  constexpr uint32_t kStageBytes = 2 * kABytes + 2 * kBBytes;
  constexpr uint32_t kSpf = FK / SK;  // stages per partial
  const uint32_t nst = a.nk * (kBK / SK);     // stages per tile
  extern __shared__ __align__(1024) uint8_t gemm_smem[];
  __shared__ GemmShared sh;
  pdl_enter();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) &
                                             ~uintptr_t(1023));

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.part_full[b], 1);
      mbar_init(&sh.part_empty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) tmem_alloc(&sh.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = sh.tmem_base;

  if (warp == 0) {
    // ---- TMA producer ----
    uint32_t issued[kStages] = {};
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      uint64_t it = first_item(a);
      GemmPiece pc;
      while (ok && next_piece<SK>(a, nst, it, pc)) {
        if (pc.skip) continue;
        const uint32_t m = pc.m, n = pc.n;
        const int row_x = int(m * kBM);
        int row_w0, row_w1;
        if constexpr (EPI == kEpiGeglu) {
          row_w0 = int(n * (kBN / 2));
          row_w1 = int(a.inter + n * (kBN / 2));
        } else {
          row_w0 = int(batch_wrow(a, m * kBM) + n * kBN);
          row_w1 = row_w0 + kBN / 2;
        }
        for (uint32_t kc = pc.s0; kc < pc.s1; ++kc, ++g) {
          const uint32_t s = g % kStages, use = g / kStages;
          if (use > 0 && !gemm_wait(&sh.empty[s], (use - 1) & 1, &sh)) {
            ok = false;
            break;
          }
          uint8_t* st = base + size_t(s) * kStageBytes;
          mbar_arrive_expect_tx(&sh.full[s], kStageBytes);
          const int k = int(kc * SK);
          tma_load_2d(st, &xh_map, &sh.full[s], k, row_x);
          tma_load_2d(st + kABytes, &xl_map, &sh.full[s], k, row_x);
          tma_load_2d(st + 2 * kABytes, &wh_map, &sh.full[s], k, row_w0);
          tma_load_2d(st + 2 * kABytes + kBBytes / 2, &wh_map, &sh.full[s], k, row_w1);
          tma_load_2d(st + 2 * kABytes + kBBytes, &wl_map, &sh.full[s], k, row_w0);
          tma_load_2d(st + 2 * kABytes + kBBytes + kBBytes / 2, &wl_map, &sh.full[s], k, row_w1);
          ++issued[s];
        }
      }
      // let this CTA's copies still in flight land before the CTA can exit
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0) mbar_wait_bounded(&sh.full[s], (issued[s] - 1) & 1, kGemmWait);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: one fresh partial per FK values of K ----
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(kBM, kBN);
      auto desc = [](uint32_t addr) {
        if constexpr (SK == 32) return smem_desc_sw128(addr);
        else return smem_desc_sw64(addr);
      };
      uint32_t g = 0, pg = 0;  // stages and partials issued
      bool ok = true;
      uint64_t it = first_item(a);
      GemmPiece pc;
      while (ok && next_piece<SK>(a, nst, it, pc)) {
        if (pc.skip) continue;
        for (uint32_t kc = pc.s0; kc < pc.s1; ++kc, ++g) {
          const uint32_t s = g % kStages, use = g / kStages;
          const uint32_t pb = pg & 1, puse = pg >> 1;
          const bool first = (kc - pc.s0) % kSpf == 0;
          if ((first && puse > 0 && !gemm_wait(&sh.part_empty[pb], (puse - 1) & 1, &sh)) ||
              !gemm_wait(&sh.full[s], use & 1, &sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tm + pb * kBN;
          const uint32_t st = smem_addr(base + size_t(s) * kStageBytes);
          const uint32_t ah = st, al = st + kABytes, bh = st + 2 * kABytes,
                         bl = st + 2 * kABytes + kBBytes;
#pragma unroll
          for (uint32_t ks = 0; ks < SK / 8; ++ks)  // x hi * w lo (starts a partial)
            mma_tf32_ss(d, desc(ah + ks * 32), desc(bl + ks * 32), idesc, !first || ks != 0);
#pragma unroll
          for (uint32_t ks = 0; ks < SK / 8; ++ks)  // x lo * w hi
            mma_tf32_ss(d, desc(al + ks * 32), desc(bh + ks * 32), idesc, 1);
#pragma unroll
          for (uint32_t ks = 0; ks < SK / 8; ++ks)  // x hi * w hi
            mma_tf32_ss(d, desc(ah + ks * 32), desc(bh + ks * 32), idesc, 1);
          mma_commit(&sh.empty[s]);  // the stage is free once these MMAs have read it
          if ((kc - pc.s0) % kSpf == kSpf - 1 || kc + 1 == pc.s1) {
            mma_commit(&sh.part_full[pb]);  // and the partial is complete
            ++pg;
          }
        }
      }
      // every MMA this thread issued has completed before TMEM is freed
      mma_commit(&sh.drain);
      mbar_wait_bounded(&sh.drain, 0, kGemmWait);
    }
    __syncwarp();
  } else if (warp >= 2) {
    // ---- epilogue: warp pairs per TMEM lane quarter, 128 columns each ----
    const uint32_t q = warp & 3;               // TMEM lane quarter
    const uint32_t half = (warp - 2) >> 2;     // which 128 of the 256 columns
    const uint32_t row = q * 32 + lane;        // token within the tile
    const uint32_t lane_off = (q * 32) << 16;
    // GeGLU: value columns [64 half, 64 half + 64) and their gate columns
    // 128 + the same; bias + act: columns [128 half, 128 half + 128).
    const uint32_t c_lo = EPI == kEpiGeglu ? 64 * half : 128 * half;
    const uint32_t c_hi = EPI == kEpiGeglu ? 128 + 64 * half : 128 * half + 64;
    float2 acc2[64];  // 128 f32 sums, added two per instruction (FADD2)
    uint32_t g = 0;
    bool ok = true;
    uint64_t it = first_item(a);
    GemmPiece pc;
    while (ok && next_piece<SK>(a, nst, it, pc)) {
      const uint32_t m = pc.m, n = pc.n;
      // a skipped piece (kCausalK) writes zeros: the SIMT kernel fills slot 0
      const uint32_t tpart = pc.skip ? 0u : (pc.s1 - pc.s0 + kSpf - 1) / kSpf;
#pragma unroll
      for (int j = 0; j < 64; ++j) acc2[j] = make_float2(0.0f, 0.0f);
      for (uint32_t kc = 0; kc < tpart; ++kc, ++g) {
        const uint32_t pb = g & 1, puse = g >> 1;
        bool got = true;
        if (lane == 0) got = gemm_wait(&sh.part_full[pb], puse & 1, &sh);
        if (!__shfl_sync(0xffffffffu, int(got), 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t src = tm + pb * kBN + lane_off;
#pragma unroll
        for (int c = 0; c < 128; c += 16) {  // one 16-column load in flight (registers)
          float v[16];
          tmem_ld16(src + (c < 64 ? c_lo + c : c_hi + c - 64), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j += 2)
            acc2[(c + j) / 2] = __fadd2_rn(acc2[(c + j) / 2], make_float2(v[j], v[j + 1]));
        }
        // this warp's reads of the partial are complete: release it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.part_empty[pb]);
      }
      float* acc = reinterpret_cast<float*>(acc2);
      if (!ok) break;
      if constexpr (EPI == kEpiBiasAct && ACT == TFX_ACT_IDENTITY && !BIAS) {
        if (a.stage_rows) {  // the whole warp, rows past the length included
          const uint32_t o0 = n * kBN + 128 * half;
          if (o0 < a.nout)
            epi_store_staged(a, m * kBM + q * 32, lane, o0, pc.slot, acc,
                             reinterpret_cast<float*>(base + size_t(kStages) * kStageBytes) +
                                 (warp - 2) * 1024);
          continue;
        }
      }
      const uint32_t t = m * kBM + row;
      if (t >= a.length) continue;
      epi_store<EPI, ACT, BIAS>(a, t, n, half, pc.slot, acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_free(tm, 512);
}

// ---- SIMT path for the tiles with non-finite (or huge) operands ----------------------
//
// The reference's arithmetic: p = bias (or 0), then p = p + x*w for i = 0,
// 1, ... (each product rounded), then the epilogue. One CTA per 128-token
// tile (most exit at once: their tile was computed on the tensor cores), one
// token per thread, blockIdx.y strides over groups of 16 outputs.
template <int EPI, int ACT>
__global__ void __launch_bounds__(128) gemm_epi_simt_kernel(const float* __restrict__ x,
                                                            const float* __restrict__ w,
                                                            GemmArgs a, uint32_t in_dim,
                                                            int force) {
  pdl_enter();
  const uint32_t m = blockIdx.x;
  if (!force && __ldcg(a.flags + m) == 0u && __ldcg(a.flags + a.mtiles) == 0u) return;
  const uint32_t t = m * kBM + threadIdx.x;
  if (t >= a.length) return;
  const float* xt = x + uint64_t(t) * in_dim;
  w += uint64_t(batch_wrow(a, t)) * in_dim;
  for (uint32_t o0 = blockIdx.y * 16; o0 < a.nout; o0 += gridDim.y * 16) {
    for (uint32_t j = o0; j < min(o0 + 16, a.nout); ++j) {
      auto proj = [&](uint32_t o) {
        float p = a.bias ? a.bias[o] : 0.0f;
        const float* wo = w + uint64_t(o) * in_dim;
        for (uint32_t i = 0; i < in_dim; ++i) p = __fadd_rn(p, __fmul_rn(xt[i], wo[i]));
        return p;
      };
      float out;
      if constexpr (EPI == kEpiGeglu) out = __fmul_rn(math::gelu_mlx(proj(j)), proj(a.inter + j));
      else out = epi_act<EPI, ACT>(proj(j));
      a.y[uint64_t(t) * a.nout + j] = out;
    }
  }
}

#include "gemm_pair.cuh"

// ---- host ----------------------------------------------------------------------------

template <int EPI, int ACT, bool BIAS, int SK, int FK>
int launch_tc(const char* op, const CUtensorMap* maps, const GemmArgs& a, const DeviceInfo& dev,
              cudaStream_t stream) {
  auto kernel = gemm_epi_tc_kernel<EPI, ACT, BIAS, SK, FK>;
  static std::once_flag once[64];
  static cudaError_t err[64];
  const int di = dev.device & 63;
  std::call_once(once[di], [&] {
    err[di] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(kGemmSmemAll));
  });
  if (err[di] != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(err[di]));
  const unsigned grid = a.causal == kCausalK
                            ? a.split.grid
                            : unsigned(std::min<uint64_t>(a.items, uint64_t(dev.sms)));
  return launch_kernel(op, kernel, dim3(grid), dim3(kGThreads), kGemmSmemAll, stream, 1, maps[0],
                       maps[1], maps[2], maps[3], a);
}

// Partial length of the tensor-core kernels. One partial per 32 values of K
// is the most accurate; per 64 is faster (one CTA: 2 %, CTA pairs: 3 %, 143.9
// -> 139.3 us on the configs[1] projection) with the error still below the
// reference's sequential sum (max 1.3e-7 of sum|x w| against 0.75e-7, and the
// reference's 3.6e-7). Default (0): the pair kernel per 64, the one-CTA
// kernel per 32. TFX_GEMM_STAGES = k32 (3: both per 32), k32f64 (1: both per
// 64), k16 (2: four stages of K 16 with 64-byte swizzle on one CTA, measured
// 5 % slower there: the MMA pipe, not the copy latency, bounds it).
int gemm_stage_layout() {
  static const int v = [] {
    const char* e = getenv("TFX_GEMM_STAGES");
    if (!e) return 0;
    const std::string s(e);
    return s == "k32f64" ? 1 : s == "k16" ? 2 : s == "k32" ? 3 : 0;
  }();
  return v;
}

// K values per stage (the inner extent of every TMA box).
int gemm_stage_k() { return gemm_stage_layout() == 2 ? 16 : 32; }

// Non-batched calls run on CTA pairs (gemm_pair_tc_kernel: 153.7 -> 139.3 us on
// the configs[1] GeGLU projection, tensor pipe 66 -> 71 % active);
// TFX_GEMM_PAIR=0 keeps them on one CTA per tile (tuning runs, and the tests
// of that kernel).
bool gemm_pair_mode() {
  static const bool v = [] {
    const char* e = getenv("TFX_GEMM_PAIR");
    return !(e && std::string(e) == "0");
  }();
  return v;
}

// TFX_GEMM_STAGE_ROWS=0: the row-major identity epilogue stores straight from
// registers (32 rows' 16 bytes per store) instead of through the staging tile.
bool gemm_stage_rows() {
  static const bool v = [] {
    const char* e = getenv("TFX_GEMM_STAGE_ROWS");
    return !(e && std::string(e) == "0");
  }();
  return v;
}

// A call runs on CTA pairs when pair mode is on and its batches (if any)
// are whole 256-token pair rows.
bool gemm_pair_call(int64_t batch_tokens, const DeviceInfo& dev) {
  return gemm_pair_mode() && dev.sms >= 2 && (batch_tokens == 0 || batch_tokens % (2 * kBM) == 0);
}

template <int EPI, int ACT, bool BIAS, int FK>
int launch_pair(const char* op, const CUtensorMap* maps, const GemmArgs& a, const DeviceInfo& dev,
                cudaStream_t stream) {
  auto kernel = gemm_pair_tc_kernel<EPI, ACT, BIAS, FK>;
  static std::once_flag once[64];
  static cudaError_t err[64];
  const int di = dev.device & 63;
  std::call_once(once[di], [&] {
    err[di] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(kGemmSmemAll));
  });
  if (err[di] != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(err[di]));
  const unsigned npairs = a.causal == kCausalK
                             ? a.split.grid
                             : unsigned(std::min<uint64_t>(a.items, uint64_t(dev.sms / 2)));
  return launch_kernel(op, kernel, dim3(2 * npairs), dim3(kGThreads), kGemmSmemAll, stream, 2,
                       maps[0], maps[1], maps[2], maps[3], a);
}

template <int EPI, int ACT, bool BIAS>
int launch_tc_layout(const char* op, const CUtensorMap* maps, const GemmArgs& a,
                     const DeviceInfo& dev, cudaStream_t stream) {
  const int layout = gemm_stage_layout();
  if (a.pair)
    return layout == 0 || layout == 1 ? launch_pair<EPI, ACT, BIAS, 64>(op, maps, a, dev, stream)
                                      : launch_pair<EPI, ACT, BIAS, 32>(op, maps, a, dev, stream);
  return layout == 1   ? launch_tc<EPI, ACT, BIAS, 32, 64>(op, maps, a, dev, stream)
         : layout == 2 ? launch_tc<EPI, ACT, BIAS, 16, 32>(op, maps, a, dev, stream)
                       : launch_tc<EPI, ACT, BIAS, 32, 32>(op, maps, a, dev, stream);
}

template <int EPI, int ACT>
int launch_all(const char* op, const float* x, const float* w, const CUtensorMap* maps,
               const GemmArgs& a, uint32_t in_dim, bool force_simt, const DeviceInfo& dev,
               cudaStream_t stream) {
  int rc = TFX_OK;
  if (!force_simt) {
    rc = a.bias ? launch_tc_layout<EPI, ACT, true>(op, maps, a, dev, stream)
                : launch_tc_layout<EPI, ACT, false>(op, maps, a, dev, stream);
    if (rc != TFX_OK) return rc;
  }
  const unsigned gy = std::min<unsigned>((a.nout + 15) / 16, 8);
  return launch_kernel(op, gemm_epi_simt_kernel<EPI, ACT>, dim3(a.mtiles, gy), dim3(128), 0,
                       stream, 1, x, w, a, in_dim, force_simt ? 1 : 0);
}

size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }

// The shared host path. nproj = rows of the weight (2I or out_dim), nout =
// outputs per token (I or out_dim).
// batch_tokens > 0 (bias + act): batched weights, batch_tokens tokens (a
// multiple of 128 dividing length) per batch of nout weight rows.
// planes (optional, batched only): x and the weight already split, {x hi,
// x lo, w hi, w lo}, row-major with in_dim (a multiple of 32) values per row:
// no split pass, no SIMT pass (the caller routes non-finite values itself).
// out_t: the token-contiguous batched output (GemmArgs::out_t).
int gemm_epilogue(const char* op, int epi, int act, const float* x, const float* w,
                  const float* bias, float* y, int64_t in_dim, int64_t nproj, int64_t nout,
                  int64_t length, cudaStream_t stream, int64_t batch_tokens = 0,
                  uint32_t causal = 0, const float* const* planes = nullptr, int out_t = 0) {
  if (nout == 0 || length == 0) return TFX_OK;  // an empty output: a no-op, as the reference
  TFX_REQUIRE(planes || x || in_dim == 0, op, "x", "null pointer");
  TFX_REQUIRE(planes || w || in_dim == 0, op, "weight", "null pointer");
  TFX_REQUIRE(!planes || (batch_tokens > 0 && in_dim > 0 && in_dim % kBK == 0 && planes[0] &&
                          planes[1] && planes[2] && planes[3]),
              op, "planes", "pre-split operands need a batched call and in_dim % 32 == 0");
  TFX_REQUIRE(y, op, "y", "null pointer");
  TFX_REQUIRE(in_dim < (int64_t(1) << 31) && nproj < (int64_t(1) << 30) &&
                  length < (int64_t(1) << 31),
              op, "shape", "extents too large for one call");
  const size_t ybytes = size_t(nout) * size_t(length) * 4;
  TFX_REQUIRE(!overlaps(x, size_t(in_dim) * size_t(length) * 4, y, ybytes), op, "y",
              "overlaps x");
  TFX_REQUIRE(!overlaps(w, size_t(in_dim) * size_t(nproj) * 4, y, ybytes), op, "y",
              "overlaps weight");
  TFX_REQUIRE(!bias || !overlaps(bias, size_t(nproj) * 4, y, ybytes), op, "y", "overlaps bias");
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;

  GemmArgs a{};
  a.y = y;
  a.bias = bias;
  a.length = uint32_t(length);
  a.nout = uint32_t(nout);
  a.inter = uint32_t(epi == kEpiGeglu ? nout : 0);
  a.mtiles = uint32_t((length + kBM - 1) / kBM);
  a.ntiles = uint32_t(epi == kEpiGeglu ? (nout + kBN / 2 - 1) / (kBN / 2)
                                       : (nout + kBN - 1) / kBN);
  a.vec4 = nout % 4 == 0 && aligned(y, 16);
  // (a split contraction with the split pass stays on one CTA per tile: there
  // the SIMT kernel's slot-0 result for a flagged tile relies on the tile's
  // other pieces being written as zeros, which only the one-CTA kernel does)
  a.pair = gemm_pair_call(batch_tokens, dev) && !(causal == kCausalK && !planes) ? 1 : 0;
  a.items = uint64_t(a.pair ? (a.mtiles + 1) / 2 : a.mtiles) * a.ntiles;
  if (batch_tokens > 0) {
    TFX_REQUIRE(epi == kEpiBiasAct && batch_tokens % kBM == 0 && length % batch_tokens == 0 &&
                    nproj == nout * (length / batch_tokens),
                op, "batch", "batched weights need whole 128-token tiles per batch");
    a.batch_tokens = uint32_t(batch_tokens);
    a.batch_wrows = uint32_t(nout);
    a.causal = causal;
    a.out_t = out_t;
    a.stage_rows = out_t || !gemm_stage_rows() ? 0 : 1;
    a.mb = uint32_t(batch_tokens / kBM);
    const uint32_t batches = uint32_t(length / batch_tokens);
    static_assert(kBN == 2 * kBM, "live score tiles assume 256-wide output tiles");
    if (causal == kCausalOut) {
      TFX_REQUIRE(nout == batch_tokens, op, "causal", "causal outputs need nout == batch_tokens");
      a.items = uint64_t(batches) *
                (a.pair ? CausalKSplit::prefix(a.mb / 2) : live_prefix(a.mb));
    } else if (causal == kCausalK) {
      TFX_REQUIRE(in_dim == batch_tokens && nout <= kBN, op, "causal",
                  "a causal contraction needs in_dim == batch_tokens and nout <= 256");
      a.split = a.pair ? causal_k_split(batches, a.mb / 2, uint32_t(dev.sms / 2), 2 * kBM)
                       : causal_k_split(batches, a.mb, uint32_t(dev.sms));
      a.slot_stride = uint64_t(length) * uint64_t(nout);
    }
  }
  TFX_REQUIRE(uint64_t(a.mtiles) * a.ntiles < (uint64_t(1) << 31), op, "shape",
              "too many tiles for one call");
  const uint64_t kp = round_up(size_t(in_dim), kBK);
  a.nk = uint32_t(kp / kBK);

  // scratch: x hi | x lo | w hi | w lo | flags, each region 1 KB aligned. Rows
  // are padded with zeros so that every 128-row box the kernel loads lies
  // inside its tensor: x to whole tiles, the weight past the last row a box
  // can start at (GeGLU: I + 128 (ntiles - 1); bias + act: 256 ntiles - 128).
  const uint64_t xrows = uint64_t(a.mtiles) * kBM;
  const uint64_t wrows = epi == kEpiGeglu ? uint64_t(nproj) + kBN / 2
                        : batch_tokens > 0
                            ? uint64_t(nproj) - uint64_t(nout) + uint64_t(a.ntiles) * kBN
                            : uint64_t(a.ntiles) * kBN;
  const size_t xbytes = planes ? 0 : round_up(kp * size_t(xrows) * 4, 1024);
  const size_t wbytes = planes ? 0 : round_up(kp * size_t(wrows) * 4, 1024);
  const size_t fbytes = round_up((size_t(a.mtiles) + 1) * 4, 1024);
  uint8_t* scratch = nullptr;
  cudaError_t e = scratch_malloc(reinterpret_cast<void**>(&scratch),
                                  2 * xbytes + 2 * wbytes + fbytes, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  }
  float* xh = reinterpret_cast<float*>(scratch);
  float* xl = reinterpret_cast<float*>(scratch + xbytes);
  float* wh = reinterpret_cast<float*>(scratch + 2 * xbytes);
  float* wl = reinterpret_cast<float*>(scratch + 2 * xbytes + wbytes);
  uint32_t* flags = reinterpret_cast<uint32_t*>(scratch + 2 * xbytes + 2 * wbytes);
  a.flags = flags;
  const bool force_simt = in_dim == 0;
  int rc = TFX_OK;
  e = cudaMemsetAsync(flags, 0, (size_t(a.mtiles) + 1) * 4, stream);
  if (e != cudaSuccess) rc = fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));

  auto prep = [&](const float* src, uint64_t cols, uint64_t cols_pad, float* hi, float* lo,
                  uint32_t* fl, uint32_t shift) {
    const uint64_t total = kp / 4 * cols_pad;
    const unsigned grid = unsigned(std::min<uint64_t>((total + 255) / 256, uint64_t(dev.sms) * 8));
    const bool v4 = in_dim % 4 == 0 && aligned(src, 16);
    return v4 ? launch_kernel(op, split_pad_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, src,
                              uint32_t(in_dim), uint32_t(cols), uint32_t(cols_pad), uint32_t(kp),
                              hi, lo, fl, shift)
              : launch_kernel(op, split_pad_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, src,
                              uint32_t(in_dim), uint32_t(cols), uint32_t(cols_pad), uint32_t(kp),
                              hi, lo, fl, shift);
  };
  CUtensorMap maps[4];
  if (rc == TFX_OK && planes) {
    // the caller's planes, at their own extents: rows past them load as zeros
    std::string why;
    for (int i = 0; rc == TFX_OK && i < 4; ++i) {
      const uint64_t rows = i < 2 ? uint64_t(length) : uint64_t(nproj);
      if (!encode_map_2d_f32(&maps[i], planes[i], kp, rows, kp, uint32_t(gemm_stage_k()), 128,
                             &why, gemm_stage_k() * 4))
        rc = fail(TFX_ERR_CUDA, op, "tensor map", why);
    }
    if (rc == TFX_OK)
      rc = launch_tc_layout<kEpiBiasAct, TFX_ACT_IDENTITY, false>(op, maps, a, dev, stream);
    cudaFreeAsync(scratch, stream);
    return rc;
  }
  if (rc == TFX_OK && !force_simt) {
    rc = prep(x, uint64_t(length), xrows, xh, xl, flags, 7);  // one flag per 128-token tile
    if (rc == TFX_OK) rc = prep(w, uint64_t(nproj), wrows, wh, wl, flags + a.mtiles, 31);
    std::string why;
    const float* bases[4] = {xh, xl, wh, wl};
    for (int i = 0; rc == TFX_OK && i < 4; ++i) {
      const uint64_t rows = i < 2 ? xrows : wrows;
      if (!encode_map_2d_f32(&maps[i], bases[i], kp, rows, kp, uint32_t(gemm_stage_k()), 128,
                             &why, gemm_stage_k() * 4))
        rc = fail(TFX_ERR_CUDA, op, "tensor map", why);
    }
  }
  if (rc == TFX_OK) {
    if (epi == kEpiGeglu)
      rc = launch_all<kEpiGeglu, 0>(op, x, w, maps, a, uint32_t(in_dim), force_simt, dev, stream);
    else if (act == TFX_ACT_GELU_ERF)
      rc = launch_all<kEpiBiasAct, TFX_ACT_GELU_ERF>(op, x, w, maps, a, uint32_t(in_dim),
                                                      force_simt, dev, stream);
    else if (act == TFX_ACT_RELU)
      rc = launch_all<kEpiBiasAct, TFX_ACT_RELU>(op, x, w, maps, a, uint32_t(in_dim), force_simt,
                                                  dev, stream);
    else
      rc = launch_all<kEpiBiasAct, TFX_ACT_IDENTITY>(op, x, w, maps, a, uint32_t(in_dim),
                                                      force_simt, dev, stream);
  }
  cudaFreeAsync(scratch, stream);
  return rc;
}

}  // namespace

// y (nout, length) = W_b^T x over batches of batch_tokens tokens: token t uses
// the weight rows of batch t / batch_tokens (weight: (in_dim, nout * batches)
// column-major, batch b's rows [b * nout, (b + 1) * nout)). Same arithmetic as
// tfx_gemm_bias_act_ff_f32 without bias and activation.
// The split of gemm_batched_f32's causal contraction (causal 2) on the
// current device: y needs split.max_pieces(length / batch_tokens) slots.
int gemm_causal_k_split(int64_t length, int64_t batch_tokens, CausalKSplit* split) {
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  // (the split of a call with pre-split operands, the only kind that runs a
  // split contraction on CTA pairs)
  const uint32_t batches = uint32_t(length / batch_tokens), mb = uint32_t(batch_tokens / kBM);
  *split = gemm_pair_call(batch_tokens, dev)
               ? causal_k_split(batches, mb / 2, uint32_t(dev.sms / 2), 2 * kBM)
               : causal_k_split(batches, mb, uint32_t(dev.sms));
  return TFX_OK;
}

// causal: 0, kCausalOut or kCausalK (GemmArgs).
int gemm_batched_f32(const char* op, const float* x, const float* w, float* y, int64_t in_dim,
                     int64_t nout, int64_t length, int64_t batch_tokens, cudaStream_t stream,
                     uint32_t causal, const float* const* planes, int out_t) {
  TFX_REQUIRE(in_dim >= 0 && nout >= 0 && length >= 0 && batch_tokens > 0 && causal <= 2, op,
              "shape", "extents must be non-negative");
  return gemm_epilogue(op, kEpiBiasAct, TFX_ACT_IDENTITY, x, w, nullptr, y, in_dim,
                       nout * (length / batch_tokens), nout, length, stream, batch_tokens, causal,
                       planes, out_t);
}

int gemm_wait_timeouts(uint32_t* count) {
  const cudaError_t err = cudaMemcpyFromSymbol(count, g_gemm_wait_timeouts, sizeof(uint32_t));
  return err == cudaSuccess ? TFX_OK
                            : fail(TFX_ERR_CUDA, "tfx", "wait timeouts", cudaGetErrorString(err));
}

}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_gemm_geglu_ff_f32(const float* x, const float* weight, const float* bias, float* y,
                          int64_t in_dim, int64_t intermediate, int64_t length,
                          tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-ext::gemm_geglu";
  TFX_REQUIRE(in_dim >= 0 && intermediate >= 0 && length >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(intermediate < (int64_t(1) << 29), op, "intermediate",
              "projected feature extent overflow");
  return gemm_epilogue(op, kEpiGeglu, TFX_ACT_IDENTITY, x, weight, bias, y, in_dim,
                       2 * intermediate, intermediate, length, stream);
}

int tfx_gemm_bias_act_ff_f32(const float* x, const float* weight, const float* bias, float* y,
                             int64_t in_dim, int64_t out_dim, int64_t length, int act,
                             tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-ext::gemm_bias";
  TFX_REQUIRE(in_dim >= 0 && out_dim >= 0 && length >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(act == TFX_ACT_IDENTITY || act == TFX_ACT_GELU_ERF || act == TFX_ACT_RELU, op,
              "act", "unknown activation " + std::to_string(act));
  return gemm_epilogue(op, kEpiBiasAct, act, x, weight, bias, y, in_dim, out_dim, out_dim,
                       length, stream);
}

}  // extern "C"
