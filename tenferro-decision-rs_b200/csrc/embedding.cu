// embedding.cu -- token embedding gather (FusedScope::embedding_rows /
// embedding_columns, crates/tenferro-ext/src/cuda_fused.rs:817-898, kernel
// fused_embedding_rows, crates/tenferro-ext/src/cuda/fused.cu:304-318).
//
// out(token t, feature f) = table(feature f, id ids[t]). Two layouts:
//   rows:    table row-major (hidden, vocab), element (f, id) at f*vocab + id;
//            out time-first (length, hidden), element (t, f) at t + length*f.
//   columns: table column-major (hidden, vocab) (each token's vector
//            contiguous), element (f, id) at f + hidden*id; out feature-first
//            (hidden, length), element (f, t) at f + hidden*t.
// The columns layout is a row copy per token (one warp, 128-bit moves); the
// rows layout reads one float per (feature, token) from scattered table
// positions, with the writes coalesced along tokens.

#include <string>
#include <vector>

#include "common.cuh"

namespace tfx {
namespace {

// Columns layout: warp per token, float4 copies when hidden % 4 == 0.
template <int VEC>
__global__ void __launch_bounds__(256) embed_columns_kernel(const float* __restrict__ table,
                                                            const int64_t* __restrict__ ids,
                                                            float* __restrict__ out,
                                                            uint32_t hidden, uint64_t vocab,
                                                            uint64_t length) {
  pdl_enter();
  const uint32_t lane = threadIdx.x & 31;
  for (uint64_t t = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; t < length;
       t += (uint64_t(gridDim.x) * blockDim.x) >> 5) {
    const int64_t id = ids[t];
    const bool ok = id >= 0 && uint64_t(id) < vocab;
    const float* src = table + (ok ? uint64_t(id) : 0) * hidden;
    float* dst = out + t * hidden;
    if constexpr (VEC == 4) {
      for (uint32_t f = lane * 4; f < hidden; f += 128) {
        float4 v = ok ? __ldg(reinterpret_cast<const float4*>(src + f))
                      : make_float4(NAN, NAN, NAN, NAN);
        *reinterpret_cast<float4*>(dst + f) = v;
      }
    } else {
      for (uint32_t f = lane; f < hidden; f += 32) dst[f] = ok ? __ldg(src + f) : NAN;
    }
  }
}

// Rows layout: one thread per (token, feature), tokens fastest.
__global__ void __launch_bounds__(256) embed_rows_kernel(const float* __restrict__ table,
                                                         const int64_t* __restrict__ ids,
                                                         float* __restrict__ out, uint64_t hidden,
                                                         uint64_t vocab, uint64_t length) {
  pdl_enter();
  const uint64_t total = hidden * length;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t f = i / length, t = i - f * length;
    const int64_t id = __ldg(ids + t);
    out[i] = id >= 0 && uint64_t(id) < vocab ? __ldg(table + f * vocab + uint64_t(id)) : NAN;
  }
}

}  // namespace

int embedding_gather(const char* op, const float* table, const int64_t* ids, float* out,
                     int64_t hidden, int64_t vocab, int64_t length, int32_t layout,
                     cudaStream_t stream) {
  TFX_REQUIRE(hidden >= 0 && vocab >= 0 && length >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(layout == TFX_EMBED_ROWS || layout == TFX_EMBED_COLUMNS, op, "layout",
              "unknown layout " + std::to_string(layout));
  if (hidden == 0 || length == 0) return TFX_OK;
  TFX_REQUIRE(vocab > 0, op, "vocab", "empty vocabulary");
  TFX_REQUIRE(table && ids && out, op, table ? (ids ? "out" : "ids") : "table", "null pointer");
  TFX_REQUIRE(hidden < (int64_t(1) << 31) && vocab < (int64_t(1) << 40), op, "shape", "too large");
  int st = TFX_OK;
  const DeviceInfo& dev = device_info(&st);
  if (st != TFX_OK) return st;
  const unsigned cap = unsigned(dev.sms) * 16;
  if (layout == TFX_EMBED_COLUMNS) {
    const uint64_t threads = uint64_t(length) * 32;
    const unsigned grid = unsigned(std::min<uint64_t>((threads + 255) / 256, cap));
    if (hidden % 4 == 0 && aligned(table, 16) && aligned(out, 16))
      return launch_kernel(op, embed_columns_kernel<4>, dim3(grid), dim3(256), 0, stream, 1, table,
                           ids, out, uint32_t(hidden), uint64_t(vocab), uint64_t(length));
    return launch_kernel(op, embed_columns_kernel<1>, dim3(grid), dim3(256), 0, stream, 1, table,
                         ids, out, uint32_t(hidden), uint64_t(vocab), uint64_t(length));
  }
  const uint64_t total = uint64_t(hidden) * uint64_t(length);
  const unsigned grid = unsigned(std::min<uint64_t>((total + 255) / 256, cap));
  return launch_kernel(op, embed_rows_kernel, dim3(grid), dim3(256), 0, stream, 1, table, ids,
                       out, uint64_t(hidden), uint64_t(vocab), uint64_t(length));
}

}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_embedding_gather_f32(const float* table, const int64_t* ids_device, float* out,
                             int64_t hidden, int64_t vocab, int64_t length, int32_t layout,
                             tfx_stream_t stream) {
  clear_error();
  return embedding_gather("tenferro-ext::embedding", table, ids_device, out, hidden, vocab,
                          length, layout, static_cast<cudaStream_t>(stream));
}

int tfx_embedding_f32(const float* table, const int64_t* ids_host, float* out, int64_t hidden,
                      int64_t vocab, int64_t length, int32_t layout, tfx_stream_t stream) {
  clear_error();
  const char* op = "tenferro-ext::embedding";
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  TFX_REQUIRE(length >= 0 && vocab >= 0, op, "shape", "extents must be non-negative");
  if (length == 0 || hidden == 0) return TFX_OK;
  TFX_REQUIRE(ids_host, op, "ids", "null pointer");
  for (int64_t t = 0; t < length; ++t)
    TFX_REQUIRE(ids_host[t] >= 0 && ids_host[t] < vocab, op, "ids",
                "token id " + std::to_string(ids_host[t]) + " at position " + std::to_string(t) +
                    " is outside the vocabulary of " + std::to_string(vocab));
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  int64_t* ids = nullptr;
  const size_t bytes = size_t(length) * sizeof(int64_t);
  cudaError_t e = scratch_malloc(reinterpret_cast<void**>(&ids), bytes, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "scratch", cudaGetErrorString(e));
  }
  e = cudaMemcpyAsync(ids, ids_host, bytes, cudaMemcpyHostToDevice, s);
  int rc = e == cudaSuccess ? TFX_OK : fail(TFX_ERR_CUDA, op, "ids", cudaGetErrorString(e));
  if (rc == TFX_OK)
    rc = embedding_gather(op, table, ids, out, hidden, vocab, length, layout, s);
  cudaFreeAsync(ids, s);
  return rc;
}

}  // extern "C"
