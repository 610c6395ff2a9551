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
                       bool swizzle128) {
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
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
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

}  // namespace

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
  *count = rms + attn;
  return TFX_OK;
}
