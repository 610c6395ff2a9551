// rms_stream.cu -- feature-last RMSNorm as a persistent, TMA-pipelined kernel.
//
// x and y are column-major (rows, width): feature d of token r sits at
// r + rows*d, so one token's features are `rows` floats apart. A tile is TOK
// consecutive tokens (32 for rows up to 512 features, else 16): one 128- or
// 64-byte run per feature. Each CTA (or CTA pair, see below) walks the tiles c, c + n, ... of
// its index c; the TMA unit copies each tile into one of STAGES
// shared-memory stages (boxes of TOK tokens x up to 256 features, completing
// on the stage's mbarrier) while the threads reduce and write an earlier
// tile. HBM sees one read and one write of the activation, the reads of
// STAGES-1 tiles are always in flight, and the load and store phases of
// different tiles overlap inside every SM -- which the register-resident
// tile kernels of norms.cu cannot do.
//
// Rows too wide for three (or at least two) 16-token stages in one SM's
// shared memory (width above ~1700) split their features over a cluster of
// two CTAs: each stages and writes its half, and the pair adds its per-token
// partial sums through distributed shared memory once per tile (rank 0's
// half first, so both CTAs compute the same scale). Measured at width 1024,
// 16-token tiles on one CTA (27.7 us for configs[2]) beat 32-token tiles on a
// pair (35.3 us: the per-tile cluster barrier), 8-token tiles (33.3 us: 32-byte
// rows), cp.async instead of TMA (27.9 us) and a ring of chunks that re-reads
// x from L2 in a second pass (29.8 us).
//
// Arithmetic per token as crates/cpu-kernels/src/lib.rs:569-577: squares
// rounded then added (no FMA contraction), scale = 1 / sqrt(sum * inv_width +
// eps), y = (x * scale) * w' with w' = 1 + w when centred. The sum is a tree
// over threads instead of the reference's sequential loop (f32 tolerance).

#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "tma.cuh"

namespace cg = cooperative_groups;

// Bounded waits in libtfx kernels that gave up (one count per CTA), per device.
static __device__ uint32_t g_wait_timeouts;

namespace tfx {

// ---- host: tensor maps ---------------------------------------------------------------

namespace {
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}
}  // namespace

bool encode_map_2d_f32(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                       uint64_t stride1, uint32_t box0, uint32_t box1, std::string* why,
                       int swizzle_bytes) {
  const auto fn = encode_fn();
  if (!fn) {
    *why = "cuTensorMapEncodeTiled is not available from the driver";
    return false;
  }
  const cuuint64_t dims[2] = {dim0, dim1};
  const cuuint64_t strides[1] = {stride1 * 4};
  const cuuint32_t box[2] = {box0, box1};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                        : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *why = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(r));
    return false;
  }
  return true;
}

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxStages = 4;
constexpr long long kWaitCycles = 1LL << 31;  // ~1 s at B200 clocks

struct StreamArgs {
  const float* w;
  float* y;
  uint32_t rows, width;
  uint32_t box1, nbox, wcta;  // features per box, boxes per stage, features per CTA
  uint32_t tiles, stages;
  float eps, inv_width;
  int centered;
};

// Shared memory: stages x [wcta][TOK] | w' [wcta] | red [kWarps][TOK] |
// part [2][TOK] | scale [TOK] | flags [2] (+ pad) | mbarriers [kMaxStages].
inline size_t stream_smem_bytes(uint32_t tok, uint32_t wcta, uint32_t stages) {
  return size_t(stages) * wcta * tok * 4 + size_t(wcta) * 4 + kWarps * tok * 4 + 3 * tok * 4 +
         16 + kMaxStages * 8;
}

// TOK tokens per tile (16 or 32); CL CTAs per cluster (1, or 2 splitting the
// features).
template <int TOK, int CL>
__global__ void __launch_bounds__(kThreads, 1)
    rms_stream_kernel(const __grid_constant__ CUtensorMap xmap, StreamArgs a) {
  constexpr int kQuads = TOK / 4;
  constexpr int kGroups = kThreads / kQuads;  // feature groups of kQuads threads
  extern __shared__ __align__(1024) unsigned char smem[];
  const uint32_t stage_floats = a.wcta * TOK;
  float* tiles_s = reinterpret_cast<float*>(smem);
  float* w_s = tiles_s + size_t(a.stages) * stage_floats;
  float* red = w_s + a.wcta;
  float* part = red + kWarps * TOK;  // [2][TOK]: this CTA's partial sums, by tile parity
  float* scale_s = part + 2 * TOK;   // [TOK]
  volatile uint32_t* flag = reinterpret_cast<volatile uint32_t*>(scale_s + TOK);  // [2]
  uint64_t* full = reinterpret_cast<uint64_t*>(scale_s + TOK + 4);

  const uint32_t rank = CL == 2 ? cg::this_cluster().block_rank() : 0;
  const uint32_t unit = blockIdx.x / CL, units = gridDim.x / CL;
  const uint32_t f_begin = rank * a.wcta;
  const uint32_t nf = a.width > f_begin ? min(a.wcta, a.width - f_begin) : 0;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t q = tid % kQuads;  // token quad of the tile: tokens 4q .. 4q+3
  const uint32_t fg = tid / kQuads;  // first local feature; then every kGroups-th
  const uint32_t n_my = a.tiles > unit ? (a.tiles - unit + units - 1) / units : 0;

  if (tid == 0) {
    for (uint32_t s = 0; s < a.stages; ++s) mbar_init(&full[s], 1);
    mbar_init_fence();
  }
  pdl_wait();  // x and w may come from the previous kernel on the stream
  for (uint32_t f = tid; f < a.wcta; f += kThreads) {
    const float wf = f < nf ? a.w[f_begin + f] : 0.0f;
    w_s[f] = a.centered ? __fadd_rn(1.0f, wf) : wf;
  }
  __syncthreads();

  auto issue = [&](uint32_t s, uint32_t k) {
    const int tok0 = int((unit + k * units) * TOK);
    float* dst = tiles_s + size_t(s) * stage_floats;
    mbar_arrive_expect_tx(&full[s], stage_floats * 4);
    for (uint32_t b = 0; b < a.nbox; ++b)
      tma_load_2d(dst + size_t(b) * a.box1 * TOK, &xmap, &full[s], tok0,
                  int(f_begin + b * a.box1));
  };
  if (tid == 0)
    for (uint32_t s = 0; s < a.stages && s < n_my; ++s) issue(s, s);
  pdl_launch_dependents();

  // Leaves after letting this CTA's loads still in flight land (bounded).
  auto drain = [&](uint32_t k) {
    if (tid == 0)
      for (uint32_t j = k; j < n_my && j < k + a.stages; ++j)
        mbar_wait_bounded(&full[j % a.stages], (j / a.stages) & 1, kWaitCycles);
    __syncthreads();
  };

  for (uint32_t k = 0; k < n_my; ++k) {
    const uint32_t s = k % a.stages, par = k & 1;
    // one thread polls (bounded), the rest wait in the CTA barrier
    const bool ok = tid != 0 || mbar_wait_bounded(&full[s], (k / a.stages) & 1, kWaitCycles);
    const bool failed = __syncthreads_or(!ok);
    if (failed && tid == 0) atomicAdd(&g_wait_timeouts, 1u);
    const float* t = tiles_s + size_t(s) * stage_floats + 4 * q;
    if (!failed) {
      // Sums of squares of the quad's 4 tokens over this thread's features.
      float2 s01 = make_float2(0.0f, 0.0f), s23 = make_float2(0.0f, 0.0f);
      for (uint32_t f = fg; f < nf; f += kGroups) {
        const float4 v = *reinterpret_cast<const float4*>(t + f * TOK);
        const float2 a01 = make_float2(v.x, v.y), a23 = make_float2(v.z, v.w);
        s01 = __fadd2_rn(s01, __fmul2_rn(a01, a01));
        s23 = __fadd2_rn(s23, __fmul2_rn(a23, a23));
      }
#pragma unroll
      for (int m = kQuads; m < 32; m <<= 1) {
        s01.x = __fadd_rn(s01.x, __shfl_xor_sync(0xffffffffu, s01.x, m));
        s01.y = __fadd_rn(s01.y, __shfl_xor_sync(0xffffffffu, s01.y, m));
        s23.x = __fadd_rn(s23.x, __shfl_xor_sync(0xffffffffu, s23.x, m));
        s23.y = __fadd_rn(s23.y, __shfl_xor_sync(0xffffffffu, s23.y, m));
      }
      if (lane < kQuads)
        *reinterpret_cast<float4*>(red + warp * TOK + 4 * lane) =
            make_float4(s01.x, s01.y, s23.x, s23.y);
    }
    __syncthreads();
    if (tid < TOK) {
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) tot = __fadd_rn(tot, red[w * TOK + tid]);
      part[par * TOK + tid] = tot;
    }
    if (tid == 0) flag[par] = failed ? 1u : 0u;
    bool stop = failed;
    const float* peer_part = part;
    if constexpr (CL == 2) {
      // Exchange partial sums (and failures) with the other CTA of the pair.
      // part[par] and flag[par] are rewritten two tiles later, after the pair
      // has met at the next exchange -- by then the peer has read them.
      cg::cluster_group cl = cg::this_cluster();
      cl.sync();
      peer_part = cl.map_shared_rank(part, rank ^ 1u);
      const volatile uint32_t* peer_flag =
          cl.map_shared_rank(const_cast<uint32_t*>(flag), rank ^ 1u);
      stop = stop || peer_flag[par] != 0;
    } else {
      __syncthreads();
    }
    if (stop) {
      drain(k);
      if constexpr (CL == 2) cg::this_cluster().sync();
      return;
    }
    if (tid < TOK) {
      float tot = part[par * TOK + tid];
      if constexpr (CL == 2) {
        const float theirs = peer_part[par * TOK + tid];
        tot = rank == 0 ? __fadd_rn(tot, theirs) : __fadd_rn(theirs, tot);
      }
      scale_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, a.inv_width), a.eps)));
    }
    __syncthreads();
    const uint32_t tok = (unit + k * units) * TOK + 4 * q;
    if (tok < a.rows) {  // rows % 4 == 0: the whole quad is in range
      const float4 sc = *reinterpret_cast<const float4*>(scale_s + 4 * q);
      float* yq = a.y + tok + size_t(f_begin) * a.rows;
      for (uint32_t f = fg; f < nf; f += kGroups) {
        const float4 v = *reinterpret_cast<const float4*>(t + f * TOK);
        const float wt = w_s[f];
        float4 o;
        o.x = __fmul_rn(__fmul_rn(v.x, sc.x), wt);
        o.y = __fmul_rn(__fmul_rn(v.y, sc.y), wt);
        o.z = __fmul_rn(__fmul_rn(v.z, sc.z), wt);
        o.w = __fmul_rn(__fmul_rn(v.w, sc.w), wt);
        *reinterpret_cast<float4*>(yq + size_t(f) * a.rows) = o;
      }
    }
    __syncthreads();  // every thread is done with stage s
    if (tid == 0 && k + a.stages < n_my) {
      fence_proxy_async_smem();
      issue(s, k + a.stages);
    }
  }
  // The peer may still read this CTA's part / flag until it passes here.
  if constexpr (CL == 2) cg::this_cluster().sync();
}

struct StreamCfg {
  uint32_t tok, cl, box1, nbox, wcta, stages;
};

// The first of (32 tokens, 1 CTA), (16, 1), (16, pair) that fits at least
// three stages, else at least two; false when none does (very wide rows).
// (A pair with 32-token tiles measured slower than one CTA with 16-token
// tiles at width 1024: the per-tile cluster barrier costs more than the
// longer rows gain.)
bool pick_cfg(uint32_t width, int smem_optin, StreamCfg* out) {
  const uint32_t cand[3][2] = {{32, 1}, {16, 1}, {16, 2}};
  for (uint32_t min_stages : {3u, 2u}) {
    for (const auto& c : cand) {
      StreamCfg g;
      g.tok = c[0];
      g.cl = c[1];
      const uint32_t per = (width + g.cl - 1) / g.cl;
      g.box1 = per >= 256 ? 256u : (per + 7) / 8 * 8;
      g.nbox = (per + g.box1 - 1) / g.box1;
      g.wcta = g.nbox * g.box1;
      g.stages = kMaxStages;
      while (g.stages >= min_stages && stream_smem_bytes(g.tok, g.wcta, g.stages) > size_t(smem_optin))
        --g.stages;
      if (g.stages >= min_stages) {
        *out = g;
        return true;
      }
    }
  }
  return false;
}

template <int TOK, int CL>
int launch_stream(const char* op, const CUtensorMap& map, const StreamArgs& a, size_t smem,
                  const DeviceInfo& dev, cudaStream_t stream) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  const int di = dev.device & 63;
  std::call_once(once[di], [&] {
    err[di] = cudaFuncSetAttribute(rms_stream_kernel<TOK, CL>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, dev.smem_optin);
  });
  if (err[di] != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(err[di]));
  const uint32_t units = std::min<uint32_t>(a.tiles, uint32_t(dev.sms) / CL);
  return launch_kernel(op, rms_stream_kernel<TOK, CL>, dim3(units * CL), dim3(kThreads), smem,
                       stream, CL, map, a);
}

// ---- ring variant: boxes through a shared-memory ring into registers -------------
//
// The stream kernel above holds each whole tile in shared memory until its
// output is written, so a stage is busy for the tile's load, reduction and
// store, and the next tile's load waits for all of it. Here one producer warp
// keeps a ring of boxes (16 tokens x 256 features, 16 KB) in flight through
// TMA, and 512 consumer threads copy each landed box into registers and hand
// its slot straight back (one mbarrier arrival per warp), so HBM reads go on
// while the consumers reduce and write. The tile being reduced lives in
// registers: 16 tokens x width, width <= 2048 (up to 16 float4 per thread).
// Tiles are dealt round-robin (tile c, c + grid, ...) so that at any moment
// the SMs read neighbouring 64-byte runs of the same features: giving each
// CTA a contiguous block of tiles measured 10 % slower at width 1024.
// Measured against the stream kernel at 16384 x 1024 (one B200, CUDA graph
// over rotating buffers): 25.7 us against 27.5 us; 32-token tiles (128-byte
// runs, 6 slots) 26.5 us; 8 or 12 slots within 1 %.

constexpr int kRingTok = 16;
constexpr int kRingConsumers = 512;
constexpr int kRingWarps = kRingConsumers / 32;
constexpr int kRingThreads = kRingConsumers + 32;  // + the producer warp
constexpr uint32_t kRingMaxSlots = 10;

struct RingArgs {
  const float* w;
  float* y;
  uint32_t rows, width;
  uint32_t box1, nbox;  // features per box (256), boxes per tile
  uint32_t tiles, slots;
  float eps, inv_width;
  int centered;
};

// Shared memory: slots x [box1][16] | w' [nbox * box1] | red [kRingWarps][16] |
// scale [16] | full, empty mbarriers [slots each].
inline size_t ring_smem_bytes(uint32_t box1, uint32_t nbox, uint32_t slots) {
  return size_t(slots) * box1 * kRingTok * 4 + size_t(nbox) * box1 * 4 +
         size_t(kRingWarps) * kRingTok * 4 + kRingTok * 4 + 2 * size_t(slots) * 8 + 8;
}

// Barrier over the consumer threads only (named barrier `id`).
__device__ __forceinline__ void consumers_sync(uint32_t id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(kRingConsumers) : "memory");
}
// The same, returning whether any consumer passed p = true.
__device__ __forceinline__ bool consumers_sync_or(uint32_t id, bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred q, o;\n\tsetp.ne.u32 q, %1, 0;\n\t"
      "barrier.cta.red.or.pred o, %2, %3, q;\n\tselp.u32 %0, 1, 0, o;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(p)), "r"(id), "r"(kRingConsumers)
      : "memory");
  return r != 0;
}

// NBMAX: boxes per tile the registers are sized for (4: width <= 1024, 8:
// width <= 2048). Consumer thread (q, fg): tokens 4q .. 4q+3 of the tile,
// local features fg and fg + 128 of every box.
template <int NBMAX>
__global__ void __launch_bounds__(kRingThreads, 1)
    rms_ring_kernel(const __grid_constant__ CUtensorMap xmap, RingArgs a) {
  constexpr int NV = 2 * NBMAX;
  extern __shared__ __align__(1024) unsigned char smem[];
  const uint32_t slot_floats = a.box1 * kRingTok;
  float* ring = reinterpret_cast<float*>(smem);
  float* w_s = ring + size_t(a.slots) * slot_floats;
  float* red = w_s + a.nbox * a.box1;
  float* scale_s = red + kRingWarps * kRingTok;
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(scale_s + kRingTok) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + a.slots;

  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t units = gridDim.x;
  const uint32_t n_my = a.tiles > blockIdx.x ? (a.tiles - blockIdx.x + units - 1) / units : 0;
  if (tid == 0) {
    for (uint32_t s = 0; s < a.slots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingWarps);
    }
    mbar_init_fence();
  }
  __syncthreads();
  pdl_enter();  // x and w may come from the previous kernel on the stream

  if (warp == kRingWarps) {  // producer: one elected lane issues every box
    if (lane == 0) {
      const uint32_t box_bytes = slot_floats * 4;
      // s, ph: slot and phase parity of the next box. A reused slot waits for
      // the release of the box issued into it one lap earlier (parity ph ^ 1).
      uint32_t issued = 0, s = 0, ph = 0;
      bool ok = true;
      for (uint32_t k = 0; k < n_my && ok; ++k) {
        const int tok0 = int((blockIdx.x + k * units) * kRingTok);
        for (uint32_t b = 0; b < a.nbox; ++b) {
          if (issued >= a.slots && !mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitCycles)) {
            atomicAdd(&g_wait_timeouts, 1u);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], box_bytes);
          tma_load_2d(ring + size_t(s) * slot_floats, &xmap, &full[s], tok0, int(b * a.box1));
          ++issued;
          if (++s == a.slots) s = 0, ph ^= 1u;
        }
      }
      // Let every copy this CTA issued land before the CTA can exit (bounded):
      // the last min(issued, slots) boxes, oldest first.
      const uint32_t back = issued < a.slots ? issued : a.slots;
      uint32_t ds = s, dph = ph;
      for (uint32_t j = 0; j < back; ++j)
        if (ds-- == 0) ds = a.slots - 1, dph ^= 1u;
      for (uint32_t j = 0; j < back; ++j) {
        mbar_wait_bounded(&full[ds], dph, kWaitCycles);
        if (++ds == a.slots) ds = 0, dph ^= 1u;
      }
    }
    return;
  }

  const uint32_t q = tid & 3, fg = tid >> 2;
  for (uint32_t f = tid; f < a.nbox * a.box1; f += kRingConsumers) {
    const float wf = f < a.width ? a.w[f] : 0.0f;
    w_s[f] = a.centered ? __fadd_rn(1.0f, wf) : wf;
  }
  consumers_sync(2);
  // Up to 1024 features the thread's weights stay in registers for all tiles.
  constexpr bool kWReg = NBMAX <= 4;
  float wr[kWReg ? NV : 1];
  if constexpr (kWReg) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const uint32_t b = uint32_t(i) >> 1, lf = fg + 128 * (uint32_t(i) & 1);
      wr[i] = b < a.nbox && lf < a.box1 ? w_s[b * a.box1 + lf] : 0.0f;
    }
  }
  uint32_t s = 0, ph = 0;  // slot and phase parity of the next box
  for (uint32_t k = 0; k < n_my; ++k) {
    float4 v[NV];
    bool bad = false;
#pragma unroll
    for (int b = 0; b < NBMAX; ++b) {
      v[2 * b] = v[2 * b + 1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (uint32_t(b) < a.nbox) {
        if (!mbar_wait_bounded(&full[s], ph, kWaitCycles)) bad = true;
        const float* t = ring + size_t(s) * slot_floats + 4 * q;
        if (fg < a.box1) v[2 * b] = *reinterpret_cast<const float4*>(t + fg * kRingTok);
        if (fg + 128 < a.box1)
          v[2 * b + 1] = *reinterpret_cast<const float4*>(t + (fg + 128) * kRingTok);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == a.slots) s = 0, ph ^= 1u;
      }
    }
    // Sums of squares of the quad's 4 tokens over this thread's features
    // (zero-filled past the width and the last token).
    float2 s01 = make_float2(0.0f, 0.0f), s23 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const float2 a01 = make_float2(v[i].x, v[i].y), a23 = make_float2(v[i].z, v[i].w);
      s01 = __fadd2_rn(s01, __fmul2_rn(a01, a01));
      s23 = __fadd2_rn(s23, __fmul2_rn(a23, a23));
    }
#pragma unroll
    for (int m = 4; m < 32; m <<= 1) {
      s01.x = __fadd_rn(s01.x, __shfl_xor_sync(0xffffffffu, s01.x, m));
      s01.y = __fadd_rn(s01.y, __shfl_xor_sync(0xffffffffu, s01.y, m));
      s23.x = __fadd_rn(s23.x, __shfl_xor_sync(0xffffffffu, s23.x, m));
      s23.y = __fadd_rn(s23.y, __shfl_xor_sync(0xffffffffu, s23.y, m));
    }
    if (lane < 4)
      *reinterpret_cast<float4*>(red + warp * kRingTok + 4 * lane) =
          make_float4(s01.x, s01.y, s23.x, s23.y);
    if (consumers_sync_or(1, bad)) {  // a copy never landed: leave (counted once)
      if (tid == 0) atomicAdd(&g_wait_timeouts, 1u);
      return;
    }
    if (tid < kRingTok) {
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < kRingWarps; ++w) tot = __fadd_rn(tot, red[w * kRingTok + tid]);
      scale_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, a.inv_width), a.eps)));
    }
    consumers_sync(2);
    const uint32_t tok = (blockIdx.x + k * units) * kRingTok + 4 * q;
    if (tok < a.rows) {  // rows % 4 == 0: the whole quad is in range
      const float4 sc = *reinterpret_cast<const float4*>(scale_s + 4 * q);
      float* yq = a.y + tok;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const uint32_t b = uint32_t(i) >> 1, lf = fg + 128 * (uint32_t(i) & 1);
        const uint32_t f = b * a.box1 + lf;
        if (b < a.nbox && lf < a.box1 && f < a.width) {
          const float wt = kWReg ? wr[kWReg ? i : 0] : w_s[f];
          float4 o;
          o.x = __fmul_rn(__fmul_rn(v[i].x, sc.x), wt);
          o.y = __fmul_rn(__fmul_rn(v[i].y, sc.y), wt);
          o.z = __fmul_rn(__fmul_rn(v[i].z, sc.z), wt);
          o.w = __fmul_rn(__fmul_rn(v[i].w, sc.w), wt);
          *reinterpret_cast<float4*>(yq + size_t(f) * a.rows) = o;
        }
      }
    }
  }
}

template <int NBMAX>
int launch_ring(const char* op, const CUtensorMap& map, const RingArgs& a, size_t smem,
                const DeviceInfo& dev, cudaStream_t stream) {
  static std::once_flag once[64];
  static cudaError_t err[64];
  const int di = dev.device & 63;
  std::call_once(once[di], [&] {
    err[di] = cudaFuncSetAttribute(rms_ring_kernel<NBMAX>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, dev.smem_optin);
  });
  if (err[di] != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(err[di]));
  const uint32_t units = std::min<uint32_t>(a.tiles, uint32_t(dev.sms));
  return launch_kernel(op, rms_ring_kernel<NBMAX>, dim3(units), dim3(kRingThreads), smem, stream,
                       1, map, a);
}

// ---- pair variant: 32-token tiles shared by a CTA pair ------------------------------
//
// The ring kernel's 16-token tiles read one 64-byte run per feature; a copy
// with that pattern already takes 24.8 us at 16384 x 1024, against 23.8 us
// for 32-token tiles (128-byte runs). One SM cannot hold a 32-token tile
// (128 KB at width 1024) in registers, and 512 such tiles over 148 SMs would
// leave a 13 % tail. So a cluster of two CTAs shares each 32-token tile: CTA
// r streams features [r*wc, r*wc + wc) (wc = half the width) through the same
// TMA box ring (boxes of 32 tokens x 128 features), reduces its per-token
// partial sums of squares, and stores them into the other CTA's shared memory
// with st.async, which completes on that CTA's mbarrier -- no cluster barrier
// per tile. Both CTAs add the two partials in rank order, so they compute the
// same scale. Two exchange slots suffice: a CTA sends tile k's partials only
// after it received the peer's partials of tile k - 1, which the peer sent
// only after it finished reading the slot of tile k - 2.

constexpr int kPairTok = 32;
constexpr uint32_t kPairBox = 128;  // features per box
constexpr uint32_t kPairMaxBoxes = 4;

struct PairArgs {
  const float* w;
  float* y;
  uint32_t rows, width;
  uint32_t wc, nbox;  // features per CTA, boxes per CTA and tile
  uint32_t tiles, slots;
  float eps, inv_width;
  int centered;
};

// Shared memory: slots x [128][32] | w' [512] | red [kRingWarps][32] |
// exchange [2][32] | scale [32] | full, empty [slots each], exchange [2] mbarriers.
inline size_t pair_smem_bytes(uint32_t slots) {
  return size_t(slots) * kPairBox * kPairTok * 4 + kPairMaxBoxes * kPairBox * 4 +
         size_t(kRingWarps) * kPairTok * 4 + 3 * kPairTok * 4 + (2 * size_t(slots) + 2) * 8 + 8;
}

__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr_local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr_local), "r"(rank));
  return r;
}
// 4 bytes into another CTA's shared memory, completing 4 bytes of transactions
// on its mbarrier at `remote_bar` (both shared::cluster addresses).
__device__ __forceinline__ void st_async_b32(uint32_t remote_addr, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                   remote_addr),
               "r"(__float_as_uint(v)), "r"(remote_bar)
               : "memory");
}

__global__ void __launch_bounds__(kRingThreads, 1)
    rms_pair_kernel(const __grid_constant__ CUtensorMap xmap, PairArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  constexpr uint32_t slot_floats = kPairBox * kPairTok;
  float* ring = reinterpret_cast<float*>(smem);
  float* w_s = ring + size_t(a.slots) * slot_floats;
  float* red = w_s + kPairMaxBoxes * kPairBox;
  float* xch = red + kRingWarps * kPairTok;  // written by the other CTA
  float* scale_s = xch + 2 * kPairTok;
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(scale_s + kPairTok) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + a.slots;
  uint64_t* xbar = empty + a.slots;

  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster.block_rank(), peer = rank ^ 1u;
  const uint32_t unit = blockIdx.x >> 1, units = gridDim.x >> 1;
  const uint32_t n_my = a.tiles > unit ? (a.tiles - unit + units - 1) / units : 0;
  const uint32_t f_begin = rank * a.wc;
  const uint32_t nf = a.width > f_begin ? min(a.wc, a.width - f_begin) : 0;
  if (tid == 0) {
    for (uint32_t s = 0; s < a.slots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingWarps);
    }
    mbar_init(&xbar[0], 1);
    mbar_init(&xbar[1], 1);
    mbar_init_fence();
  }
  cluster.sync();  // both CTAs' mbarriers exist before any remote arrival
  pdl_wait();      // x and w may come from the previous kernel on the stream

  if (warp == kRingWarps) {  // producer: one elected lane issues every box
    if (lane == 0) {
      const uint32_t box_bytes = slot_floats * 4;
      uint32_t issued = 0, s = 0, ph = 0;
      bool ok = true;
      for (uint32_t k = 0; k < n_my && ok; ++k) {
        const int tok0 = int((unit + k * units) * kPairTok);
        for (uint32_t b = 0; b < a.nbox; ++b) {
          if (issued >= a.slots && !mbar_wait_bounded(&empty[s], ph ^ 1u, kWaitCycles)) {
            atomicAdd(&g_wait_timeouts, 1u);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], box_bytes);
          tma_load_2d(ring + size_t(s) * slot_floats, &xmap, &full[s], tok0,
                      int(f_begin + b * kPairBox));
          ++issued;
          if (++s == a.slots) s = 0, ph ^= 1u;
        }
      }
      // every copy this CTA issued lands before the CTA can exit (bounded)
      const uint32_t back = issued < a.slots ? issued : a.slots;
      uint32_t ds = s, dph = ph;
      for (uint32_t j = 0; j < back; ++j)
        if (ds-- == 0) ds = a.slots - 1, dph ^= 1u;
      for (uint32_t j = 0; j < back; ++j) {
        mbar_wait_bounded(&full[ds], dph, kWaitCycles);
        if (++ds == a.slots) ds = 0, dph ^= 1u;
      }
    }
    __syncwarp();
  } else {
    // consumer thread (q, fg): tokens 4q .. 4q+3 of the tile, local features
    // fg and fg + 64 of every box
    const uint32_t q = tid & 7, fg = tid >> 3;
    for (uint32_t f = tid; f < kPairMaxBoxes * kPairBox; f += kRingConsumers) {
      const float wf = f < nf ? a.w[f_begin + f] : 0.0f;
      w_s[f] = a.centered ? __fadd_rn(1.0f, wf) : wf;
    }
    consumers_sync(2);
    constexpr int NV = 2 * kPairMaxBoxes;
    float wr[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) wr[i] = w_s[(i >> 1) * kPairBox + fg + 64 * (i & 1)];
    const uint32_t xch_peer = map_to_rank(smem_addr(xch), peer);
    const uint32_t xbar_peer = map_to_rank(smem_addr(xbar), peer);
    uint32_t s = 0, ph = 0;
    for (uint32_t k = 0; k < n_my; ++k) {
      float4 v[NV];
      bool bad = false;
#pragma unroll
      for (int b = 0; b < int(kPairMaxBoxes); ++b) {
        v[2 * b] = v[2 * b + 1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (uint32_t(b) < a.nbox) {
          if (!mbar_wait_bounded(&full[s], ph, kWaitCycles)) bad = true;
          const float* t = ring + size_t(s) * slot_floats + 4 * q;
          const uint32_t lf = b * kPairBox + fg;
          if (lf < nf) v[2 * b] = *reinterpret_cast<const float4*>(t + fg * kPairTok);
          if (lf + 64 < nf) v[2 * b + 1] = *reinterpret_cast<const float4*>(t + (fg + 64) * kPairTok);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          if (++s == a.slots) s = 0, ph ^= 1u;
        }
      }
      float2 s01 = make_float2(0.0f, 0.0f), s23 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const float2 a01 = make_float2(v[i].x, v[i].y), a23 = make_float2(v[i].z, v[i].w);
        s01 = __fadd2_rn(s01, __fmul2_rn(a01, a01));
        s23 = __fadd2_rn(s23, __fmul2_rn(a23, a23));
      }
#pragma unroll
      for (int m = 8; m < 32; m <<= 1) {
        s01.x = __fadd_rn(s01.x, __shfl_xor_sync(0xffffffffu, s01.x, m));
        s01.y = __fadd_rn(s01.y, __shfl_xor_sync(0xffffffffu, s01.y, m));
        s23.x = __fadd_rn(s23.x, __shfl_xor_sync(0xffffffffu, s23.x, m));
        s23.y = __fadd_rn(s23.y, __shfl_xor_sync(0xffffffffu, s23.y, m));
      }
      if (lane < 8)
        *reinterpret_cast<float4*>(red + warp * kPairTok + 4 * lane) =
            make_float4(s01.x, s01.y, s23.x, s23.y);
      if (consumers_sync_or(1, bad)) {  // a copy never landed: leave (counted once)
        if (tid == 0) atomicAdd(&g_wait_timeouts, 1u);
        break;
      }
      // this CTA's partial for token tid, to the other CTA's slot k & 1
      float own = 0.0f;
      const uint32_t xs = k & 1u;
      if (tid < kPairTok) {
#pragma unroll
        for (int w = 0; w < kRingWarps; ++w) own = __fadd_rn(own, red[w * kPairTok + tid]);
        if (tid == 0) mbar_arrive_expect_tx(&xbar[xs], kPairTok * 4);
        st_async_b32(xch_peer + (xs * kPairTok + tid) * 4, own, xbar_peer + xs * 8);
      }
      // each reader observes the exchange mbarrier itself (the peer's async
      // stores are visible to the threads that see the phase complete)
      bool late = false;
      if (tid < kPairTok) late = !mbar_wait_bounded(&xbar[xs], (k >> 1) & 1u, kWaitCycles);
      if (consumers_sync_or(3, late)) {  // the other CTA's partials never came
        if (tid == 0) atomicAdd(&g_wait_timeouts, 1u);
        break;
      }
      if (tid < kPairTok) {
        const float other = xch[xs * kPairTok + tid];
        const float tot = rank == 0 ? __fadd_rn(own, other) : __fadd_rn(other, own);
        scale_s[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, a.inv_width), a.eps)));
      }
      consumers_sync(2);
      const uint32_t tok = (unit + k * units) * kPairTok + 4 * q;
      if (tok < a.rows) {  // rows % 4 == 0: the whole quad is in range
        const float4 sc = *reinterpret_cast<const float4*>(scale_s + 4 * q);
        float* yq = a.y + tok;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const uint32_t lf = (uint32_t(i) >> 1) * kPairBox + fg + 64 * (uint32_t(i) & 1);
          if (uint32_t(i >> 1) < a.nbox && lf < nf) {
            float4 o;
            o.x = __fmul_rn(__fmul_rn(v[i].x, sc.x), wr[i]);
            o.y = __fmul_rn(__fmul_rn(v[i].y, sc.y), wr[i]);
            o.z = __fmul_rn(__fmul_rn(v[i].z, sc.z), wr[i]);
            o.w = __fmul_rn(__fmul_rn(v[i].w, sc.w), wr[i]);
            *reinterpret_cast<float4*>(yq + size_t(f_begin + lf) * a.rows) = o;
          }
        }
      }
    }
  }
  // neither CTA leaves while the other may still store into its shared memory
  cluster.sync();
}

}  // namespace

// Ring RMSNorm; 1 when the shape or alignment is not covered (nothing
// launched), else a status. Covers rows % 4 == 0, 16-byte aligned x and y,
// rows < 2^31 and 512 < width <= 2048.
int rms_ring(const char* op, const float* x, const float* w, float* y, uint32_t rows,
             uint32_t width, int centered, float eps, float inv_width, cudaStream_t stream) {
  if (rows % 4 != 0 || rows >= (1u << 31) || !aligned(x, 16) || !aligned(y, 16)) return 1;
  if (width <= 512 || width > 2048) return 1;
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  RingArgs a;
  a.box1 = 256;
  a.nbox = (width + a.box1 - 1) / a.box1;
  a.slots = kRingMaxSlots;
  while (a.slots > 2 && ring_smem_bytes(a.box1, a.nbox, a.slots) > size_t(dev.smem_optin))
    --a.slots;
  if (ring_smem_bytes(a.box1, a.nbox, a.slots) > size_t(dev.smem_optin)) return 1;
  CUtensorMap map;
  std::string why;
  if (!encode_map_2d_f32(&map, x, rows, width, rows, kRingTok, a.box1, &why))
    return fail(TFX_ERR_CUDA, op, "tensor map", why);
  a.w = w;
  a.y = y;
  a.rows = rows;
  a.width = width;
  a.tiles = (rows + kRingTok - 1) / kRingTok;
  a.eps = eps;
  a.inv_width = inv_width;
  a.centered = centered;
  const size_t smem = ring_smem_bytes(a.box1, a.nbox, a.slots);
  if (a.nbox <= 4) return launch_ring<4>(op, map, a, smem, dev, stream);
  return launch_ring<8>(op, map, a, smem, dev, stream);
}

// Pair RMSNorm (32-token tiles shared by a CTA pair); 1 when the shape or
// alignment is not covered (nothing launched), else a status. Covers rows %
// 4 == 0, 16-byte aligned x and y, rows < 2^31 and 512 < width <= 1024.
int rms_pair(const char* op, const float* x, const float* w, float* y, uint32_t rows,
             uint32_t width, int centered, float eps, float inv_width, cudaStream_t stream) {
  if (rows % 4 != 0 || rows >= (1u << 31) || !aligned(x, 16) || !aligned(y, 16)) return 1;
  if (width <= 512 || width > 2 * kPairMaxBoxes * kPairBox) return 1;
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  PairArgs a;
  a.wc = (width + 1) / 2;
  a.nbox = (a.wc + kPairBox - 1) / kPairBox;
  a.slots = kRingMaxSlots;
  while (a.slots > 2 && pair_smem_bytes(a.slots) > size_t(dev.smem_optin)) --a.slots;
  if (pair_smem_bytes(a.slots) > size_t(dev.smem_optin) || dev.sms < 2) return 1;
  CUtensorMap map;
  std::string why;
  if (!encode_map_2d_f32(&map, x, rows, width, rows, kPairTok, kPairBox, &why))
    return fail(TFX_ERR_CUDA, op, "tensor map", why);
  a.w = w;
  a.y = y;
  a.rows = rows;
  a.width = width;
  a.tiles = (rows + kPairTok - 1) / kPairTok;
  a.eps = eps;
  a.inv_width = inv_width;
  a.centered = centered;
  const size_t smem = pair_smem_bytes(a.slots);
  static std::once_flag once[64];
  static cudaError_t err[64];
  const int di = dev.device & 63;
  std::call_once(once[di], [&] {
    err[di] = cudaFuncSetAttribute(rms_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   dev.smem_optin);
  });
  if (err[di] != cudaSuccess) return fail(TFX_ERR_CUDA, op, "launch", cudaGetErrorString(err[di]));
  const uint32_t units = std::min<uint32_t>(a.tiles, uint32_t(dev.sms) / 2);
  return launch_kernel(op, rms_pair_kernel, dim3(2 * units), dim3(kRingThreads), smem, stream, 2,
                       map, a);
}

// Streaming RMSNorm; 1 when the shape or alignment is not covered (nothing
// launched), else a status. Needs rows % 4 == 0, 16-byte aligned x and y,
// rows < 2^31 and two stages of a tile in shared memory (width up to about
// 3300 features).
int rms_stream(const char* op, const float* x, const float* w, float* y, uint32_t rows,
               uint32_t width, int centered, float eps, float inv_width, cudaStream_t stream) {
  if (rows % 4 != 0 || rows >= (1u << 31) || !aligned(x, 16) || !aligned(y, 16)) return 1;
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  StreamCfg g;
  if (!pick_cfg(width, dev.smem_optin, &g)) return 1;
  CUtensorMap map;
  std::string why;
  if (!encode_map_2d_f32(&map, x, rows, width, rows, g.tok, g.box1, &why))
    return fail(TFX_ERR_CUDA, op, "tensor map", why);
  StreamArgs a;
  a.w = w;
  a.y = y;
  a.rows = rows;
  a.width = width;
  a.box1 = g.box1;
  a.nbox = g.nbox;
  a.wcta = g.wcta;
  a.tiles = (rows + g.tok - 1) / g.tok;
  a.stages = g.stages;
  a.eps = eps;
  a.inv_width = inv_width;
  a.centered = centered;
  const size_t smem = stream_smem_bytes(g.tok, g.wcta, g.stages);
  if (g.tok == 32) return launch_stream<32, 1>(op, map, a, smem, dev, stream);
  if (g.cl == 1) return launch_stream<16, 1>(op, map, a, smem, dev, stream);
  return launch_stream<16, 2>(op, map, a, smem, dev, stream);
}

}  // namespace tfx

extern "C" int tfx_wait_timeouts(uint32_t* count) {
  tfx::clear_error();
  if (!count) return tfx::fail(TFX_ERR_INVALID_ARGUMENT, "tfx", "count", "null pointer");
  int st = TFX_OK;
  tfx::device_info(&st);
  if (st != TFX_OK) return st;
  uint32_t rms = 0, attn = 0;
  const cudaError_t err = cudaMemcpyFromSymbol(&rms, g_wait_timeouts, sizeof(uint32_t));
  if (err != cudaSuccess)
    return tfx::fail(TFX_ERR_CUDA, "tfx", "wait timeouts", cudaGetErrorString(err));
  st = tfx::attention_wait_timeouts(&attn);
  if (st != TFX_OK) return st;
  uint32_t gemm = 0;
  st = tfx::gemm_wait_timeouts(&gemm);
  if (st != TFX_OK) return st;
  *count = rms + attn + gemm;
  return TFX_OK;
}
