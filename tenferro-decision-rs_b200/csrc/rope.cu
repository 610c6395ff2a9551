// rope.cu -- rotary position embedding with pairs (i, i + rotary_dim/2)
// (crates/tenferro-infer/src/rope.rs:68-113) on a strided activation.
//
// Channel-contiguous layouts (stride_feat == 1, e.g. the q and k blocks of a
// feature-first qkv (3*hidden, length, batch)) take a vector kernel: a thread
// rotates 4 consecutive pairs with four 128-bit loads (x_i, x_{i+half} and the
// two table rows, which stay in L1/L2) and two 128-bit stores. Other layouts
// (e.g. the (..., seq, head) column-major tensors of tenferro-infer, whose
// leading axes are contiguous) take a scalar kernel ordered so that
// consecutive threads touch consecutive addresses.

#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"

namespace tfx {
namespace {

struct RopeArgs {
  int64_t n_vec, seq, batch, head_dim, rotary_dim, half;
  int64_t s_vec, s_pos, s_batch, s_feat;
};

// y1 = x1*c - x2*s, y2 = x1*s + x2*c, each product rounded (rope.rs:103-110).
__device__ __forceinline__ void rotate(float x1, float x2, float c, float s, float& y1,
                                       float& y2) {
  y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  y2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
}

// Units per vector: half/4 rotation units, then (copy ? tail/4 : 0) copy units.
// A thread takes U units per iteration (t, t + step, ...) and issues all their
// loads before any arithmetic, so U x 32 bytes of the activation are in flight
// per thread (the tables stay in L1 / L2). Measured on the chain's q, k
// (402.7 MB): U = 1 70.1 us, U = 2 67.5 us, U = 4 66.2 us (the default;
// TFX_ROPE_UNROLL=1|2|4 overrides it for tuning runs).
template <int U>
__global__ void __launch_bounds__(256) rope_vec_kernel(const float* x, float* y,
                                                       const float* __restrict__ cos_t,
                                                       const float* __restrict__ sin_t,
                                                       RopeArgs a, uint64_t total,
                                                       FastDiv units_div, FastDiv vec_div,
                                                       FastDiv seq_div, uint32_t rot_units) {
  pdl_enter();
  const uint64_t step = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t t0 = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t0 < total;
       t0 += U * step) {
    int64_t base[U], off[U];
    bool rot[U], live[U];
    float4 x1[U], x2[U], c[U], sn[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const uint64_t t = t0 + k * step;
      live[k] = t < total;
      if (!live[k]) continue;
      const uint32_t tt = uint32_t(t);
      const uint32_t vi = units_div.div(tt);
      const uint32_t u = tt - vi * units_div.d;
      const uint32_t bp = vec_div.div(vi);
      const uint32_t v = vi - bp * vec_div.d;
      const uint32_t b = seq_div.div(bp);
      const uint32_t p = bp - b * seq_div.d;
      base[k] = int64_t(v) * a.s_vec + int64_t(p) * a.s_pos + int64_t(b) * a.s_batch;
      rot[k] = u < rot_units;
      if (rot[k]) {
        off[k] = int64_t(u) * 4;
        x1[k] = ld_stream(reinterpret_cast<const float4*>(x + base[k] + off[k]));
        x2[k] = ld_stream(reinterpret_cast<const float4*>(x + base[k] + a.half + off[k]));
        c[k] = __ldg(reinterpret_cast<const float4*>(cos_t + int64_t(p) * a.half + off[k]));
        sn[k] = __ldg(reinterpret_cast<const float4*>(sin_t + int64_t(p) * a.half + off[k]));
      } else {
        off[k] = a.rotary_dim + int64_t(u - rot_units) * 4;
        x1[k] = ld_stream(reinterpret_cast<const float4*>(x + base[k] + off[k]));
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      if (!live[k]) continue;
      if (rot[k]) {
        float4 y1, y2;
        rotate(x1[k].x, x2[k].x, c[k].x, sn[k].x, y1.x, y2.x);
        rotate(x1[k].y, x2[k].y, c[k].y, sn[k].y, y1.y, y2.y);
        rotate(x1[k].z, x2[k].z, c[k].z, sn[k].z, y1.z, y2.z);
        rotate(x1[k].w, x2[k].w, c[k].w, sn[k].w, y1.w, y2.w);
        *reinterpret_cast<float4*>(y + base[k] + off[k]) = y1;
        *reinterpret_cast<float4*>(y + base[k] + a.half + off[k]) = y2;
      } else {
        *reinterpret_cast<float4*>(y + base[k] + off[k]) = x1[k];
      }
    }
  }
}

// One thread per (pair or copied channel, vector, position, batch). With
// vec_fastest the vector index varies fastest (contiguous leading axes).
__global__ void __launch_bounds__(256) rope_scalar_kernel(const float* x, float* y,
                                                          const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t,
                                                          RopeArgs a, int64_t work_per_vec,
                                                          int vec_fastest, uint64_t total) {
  pdl_enter();
  const uint64_t step = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += step) {
    uint64_t r = t;
    int64_t v, u;
    if (vec_fastest) {
      v = int64_t(r % uint64_t(a.n_vec));
      r /= uint64_t(a.n_vec);
      u = int64_t(r % uint64_t(work_per_vec));
      r /= uint64_t(work_per_vec);
    } else {
      u = int64_t(r % uint64_t(work_per_vec));
      r /= uint64_t(work_per_vec);
      v = int64_t(r % uint64_t(a.n_vec));
      r /= uint64_t(a.n_vec);
    }
    const int64_t p = int64_t(r % uint64_t(a.seq));
    const int64_t b = int64_t(r / uint64_t(a.seq));
    const int64_t base = v * a.s_vec + p * a.s_pos + b * a.s_batch;
    if (u < a.half) {
      const float x1 = x[base + u * a.s_feat];
      const float x2 = x[base + (u + a.half) * a.s_feat];
      float y1, y2;
      rotate(x1, x2, __ldg(cos_t + p * a.half + u), __ldg(sin_t + p * a.half + u), y1, y2);
      y[base + u * a.s_feat] = y1;
      y[base + (u + a.half) * a.s_feat] = y2;
    } else {
      const int64_t j = a.rotary_dim + (u - a.half);
      y[base + j * a.s_feat] = x[base + j * a.s_feat];
    }
  }
}

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" int tfx_rope_pairhalf_f32(const float* x, float* y, const float* cos_table,
                                     const float* sin_table, const tfx_rope_desc* d,
                                     tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-infer::rope";
  TFX_REQUIRE(d, op, "desc", "null pointer");
  TFX_REQUIRE(d->n_vec >= 0 && d->seq >= 0 && d->batch >= 0 && d->head_dim >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(d->rotary_dim > 0 && d->rotary_dim % 2 == 0, op, "rotary_dim",
              "rotary width must be a positive even number, got " + std::to_string(d->rotary_dim));
  TFX_REQUIRE(d->rotary_dim <= d->head_dim, op, "rotary_dim",
              "rotary_dim " + std::to_string(d->rotary_dim) + " exceeds head dimension " +
                  std::to_string(d->head_dim));
  if (d->n_vec == 0 || d->seq == 0 || d->batch == 0) return TFX_OK;
  TFX_REQUIRE(x && y, op, x ? "y" : "x", "null pointer");
  TFX_REQUIRE(cos_table && sin_table, op, "tables", "null pointer");
  TFX_REQUIRE(d->stride_vec >= 0 && d->stride_pos >= 0 && d->stride_batch >= 0 &&
                  d->stride_feat > 0,
              op, "strides", "strides must be non-negative (stride_feat positive)");
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;

  RopeArgs a;
  a.n_vec = d->n_vec;
  a.seq = d->seq;
  a.batch = d->batch;
  a.head_dim = d->head_dim;
  a.rotary_dim = d->rotary_dim;
  a.half = d->rotary_dim / 2;
  a.s_vec = d->stride_vec;
  a.s_pos = d->stride_pos;
  a.s_batch = d->stride_batch;
  a.s_feat = d->stride_feat;
  const bool copy_tail = x != y && d->rotary_dim < d->head_dim;
  const int64_t tail = copy_tail ? d->head_dim - d->rotary_dim : 0;
  const int64_t vectors = d->n_vec * d->seq * d->batch;

  const bool vec = a.s_feat == 1 && a.half % 4 == 0 && tail % 4 == 0 && a.s_vec % 4 == 0 &&
                   a.s_pos % 4 == 0 && a.s_batch % 4 == 0 && aligned(x, 16) && aligned(y, 16) &&
                   aligned(cos_table, 16) && aligned(sin_table, 16);
  if (vec) {
    const int64_t units = a.half / 4 + tail / 4;
    const int64_t total = vectors * units;
    if (total < (int64_t(1) << 32) && vectors < (int64_t(1) << 32)) {
      const uint64_t grid =
          std::min<uint64_t>((uint64_t(total) + 255) / 256, uint64_t(dev.sms) * 8);
      static const int unroll = [] {
        const char* e = getenv("TFX_ROPE_UNROLL");
        return e ? std::max(1, std::min(4, atoi(e))) : 4;
      }();
      auto go = [&](auto kernel) {
        return launch_kernel(op, kernel, dim3(unsigned(grid)), dim3(256), 0, stream, 1, x, y,
                             cos_table, sin_table, a, uint64_t(total), FastDiv(uint32_t(units)),
                             FastDiv(uint32_t(a.n_vec)), FastDiv(uint32_t(a.seq)),
                             uint32_t(a.half / 4));
      };
      if (unroll >= 4) return go(rope_vec_kernel<4>);
      if (unroll >= 2) return go(rope_vec_kernel<2>);
      return go(rope_vec_kernel<1>);
    }
  }
  const int64_t work = a.half + tail;
  const uint64_t total = uint64_t(vectors) * uint64_t(work);
  const int vec_fastest = a.s_vec < a.s_feat ? 1 : 0;
  const uint64_t grid = std::min<uint64_t>((total + 255) / 256, uint64_t(dev.sms) * 8);
  return launch_kernel(op, rope_scalar_kernel, dim3(unsigned(grid)), dim3(256), 0, stream, 1, x, y,
                       cos_table, sin_table, a, work, vec_fastest, total);
}
