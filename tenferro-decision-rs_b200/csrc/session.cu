// session.cu -- the extension ops on HOST buffers, the form in which the
// reference's CPU sessions hand them tensors (TensorRead of host memory,
// crates/tenferro-ext/src/*.rs execute_*_in_session). A session owns one GPU's
// streams and staging memory; every call splits its token axis into chunks
// and pipelines them over three streams -- chunk k's host-to-device copy,
// chunk k-1's kernel and chunk k-2's device-to-host copy run at the same time
// on the two copy engines and the SMs -- and returns once the host outputs are
// written. Pinned host buffers give fully asynchronous copies; pageable ones
// work too (the runtime stages them), at lower throughput.
//
// Staging memory is allocated when a call first needs more than the session
// holds and is kept for later calls; tfx_session_destroy frees it.

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "chunk_plan.h"
#include "common.cuh"
#include "internal.h"

struct tfx_session {
  static constexpr int kMaxStreams = 8;
  int device = 0;
  int nstreams = 3;  // streams (and staging slots) a call's chunks rotate over
  cudaStream_t streams[kMaxStreams] = {};
  cudaEvent_t params_ready = nullptr;
  char* slot[kMaxStreams] = {};
  size_t slot_cap = 0;
  char* params = nullptr;
  size_t params_cap = 0;
  int64_t chunk_bytes = int64_t(32) << 20;
  std::mutex mu;
  std::map<std::tuple<double, int64_t, int64_t>, std::pair<std::vector<float>, std::vector<float>>>
      tables;
};

namespace tfx {
namespace {

int cuda_fail(const char* op, const char* what, cudaError_t err) {
  return fail(TFX_ERR_CUDA, op, what,
              std::string(cudaGetErrorName(err)) + ": " + cudaGetErrorString(err));
}

// Makes the session's device current for the call and restores the caller's.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    ok_ = cudaGetDevice(&prev_) == cudaSuccess && cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = -1;
  bool ok_ = false;
};

int sync_all(tfx_session* s, const char* op) {
  for (int i = 0; i < s->nstreams; ++i) {
    const cudaError_t err = cudaStreamSynchronize(s->streams[i]);
    if (err != cudaSuccess) return cuda_fail(op, "stream", err);
  }
  return TFX_OK;
}

int ensure_slots(tfx_session* s, size_t bytes, const char* op) {
  if (bytes <= s->slot_cap) return TFX_OK;
  int rc = sync_all(s, op);
  if (rc != TFX_OK) return rc;
  for (auto& p : s->slot) {
    if (p) cudaFree(p);
    p = nullptr;
  }
  s->slot_cap = 0;
  for (int i = 0; i < s->nstreams; ++i) {
    const cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&s->slot[i]), bytes);
    if (err != cudaSuccess) return cuda_fail(op, "staging", err);
  }
  s->slot_cap = bytes;
  return TFX_OK;
}

int ensure_params(tfx_session* s, size_t bytes, const char* op) {
  if (bytes <= s->params_cap) return TFX_OK;
  int rc = sync_all(s, op);
  if (rc != TFX_OK) return rc;
  if (s->params) cudaFree(s->params);
  s->params = nullptr;
  s->params_cap = 0;
  const cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&s->params), bytes);
  if (err != cudaSuccess) return cuda_fail(op, "params", err);
  s->params_cap = bytes;
  return TFX_OK;
}

// Uploads small per-call parameters (weights, tables, masks) into the params
// area on stream 0 and makes the other streams wait for them. Each entry is
// placed at a 256-byte aligned offset; returns the device addresses.
struct Param {
  const void* host;
  size_t bytes;
};

int upload_params(tfx_session* s, const char* op, std::initializer_list<Param> in,
                  std::vector<const void*>* out) {
  size_t total = 0;
  for (const Param& p : in) total += (p.bytes + 255) / 256 * 256;
  if (total == 0) {
    out->assign(in.size(), nullptr);
    return TFX_OK;
  }
  int rc = ensure_params(s, total, op);
  if (rc != TFX_OK) return rc;
  size_t off = 0;
  out->clear();
  for (const Param& p : in) {
    if (!p.host || p.bytes == 0) {
      out->push_back(nullptr);
      continue;
    }
    char* dst = s->params + off;
    const cudaError_t err =
        cudaMemcpyAsync(dst, p.host, p.bytes, cudaMemcpyHostToDevice, s->streams[0]);
    if (err != cudaSuccess) return cuda_fail(op, "params", err);
    out->push_back(dst);
    off += (p.bytes + 255) / 256 * 256;
  }
  cudaError_t err = cudaEventRecord(s->params_ready, s->streams[0]);
  if (err != cudaSuccess) return cuda_fail(op, "params", err);
  for (int k = 1; k < s->nstreams; ++k) {
    err = cudaStreamWaitEvent(s->streams[k], s->params_ready, 0);
    if (err != cudaSuccess) return cuda_fail(op, "params", err);
  }
  return TFX_OK;
}

int h2d(const char* op, void* dst, const void* src, size_t bytes, cudaStream_t st) {
  const cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st);
  return err == cudaSuccess ? TFX_OK : cuda_fail(op, "copy to device", err);
}

int d2h(const char* op, void* dst, const void* src, size_t bytes, cudaStream_t st) {
  const cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st);
  return err == cudaSuccess ? TFX_OK : cuda_fail(op, "copy to host", err);
}

// Runs the call's chunks (plan_chunks; at most per_chunk units each, so each
// fits a slot sized for per_chunk) round-robin over the session's streams;
// stage() gets (first unit, units, stream, slot) and enqueues copies and the
// kernel.
template <class Stage>
int pipeline(tfx_session* s, const char* op, int64_t units, int64_t per_chunk, Stage stage,
             int64_t align = 1) {
  int rc = TFX_OK;
  int64_t k = 0, u0 = 0;
  for (const int64_t n : plan_chunks(units, per_chunk, align)) {
    if (rc != TFX_OK) break;
    const int idx = int(k % s->nstreams);
    rc = stage(u0, n, s->streams[idx], s->slot[idx]);
    u0 += n;
    ++k;
  }
  const int rc2 = sync_all(s, op);
  return rc != TFX_OK ? rc : rc2;
}

// Units per chunk for `unit_bytes` of staging per unit (input + output).
int64_t units_per_chunk(const tfx_session* s, int64_t unit_bytes, int64_t align = 1) {
  int64_t n = std::max<int64_t>(1, s->chunk_bytes / std::max<int64_t>(1, unit_bytes));
  if (n > align) n = n / align * align;
  return n;
}

#define TFX_SESSION_ENTER(op)                                              \
  clear_error();                                                           \
  TFX_REQUIRE(s, op, "session", "null session");                          \
  std::lock_guard<std::mutex> lock(s->mu);                                 \
  DeviceGuard guard(s->device);                                            \
  if (!guard.ok()) return fail(TFX_ERR_CUDA, op, "device", "cannot select the session's device")

}  // namespace
}  // namespace tfx

using namespace tfx;

extern "C" {

int tfx_session_create(int device, tfx_session** out) {
  clear_error();
  const char* op = "tfx_session";
  TFX_REQUIRE(out, op, "out", "null pointer");
  *out = nullptr;
  int count = 0;
  cudaError_t err = cudaGetDeviceCount(&count);
  if (err != cudaSuccess) return cuda_fail(op, "device", err);
  TFX_REQUIRE(device >= 0 && device < count, op, "device",
              "no CUDA device " + std::to_string(device));
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(TFX_ERR_CUDA, op, "device", "cannot select the device");
  int st = TFX_OK;
  device_info(&st);
  if (st != TFX_OK) return st;
  auto* s = new tfx_session();
  s->device = device;
  if (const char* e = getenv("TFX_SESSION_STREAMS"))  // tuning runs only
    s->nstreams = std::max(2, std::min(tfx_session::kMaxStreams, atoi(e)));
  for (int i = 0; i < s->nstreams; ++i) {
    err = cudaStreamCreateWithFlags(&s->streams[i], cudaStreamNonBlocking);
    if (err != cudaSuccess) {
      tfx_session_destroy(s);
      return cuda_fail(op, "stream", err);
    }
  }
  err = cudaEventCreateWithFlags(&s->params_ready, cudaEventDisableTiming);
  if (err != cudaSuccess) {
    tfx_session_destroy(s);
    return cuda_fail(op, "event", err);
  }
  *out = s;
  return TFX_OK;
}

int tfx_session_destroy(tfx_session* s) {
  clear_error();
  if (!s) return TFX_OK;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    DeviceGuard guard(s->device);
    for (auto st : s->streams)
      if (st) cudaStreamSynchronize(st);
    for (auto& p : s->slot)
      if (p) cudaFree(p);
    if (s->params) cudaFree(s->params);
    if (s->params_ready) cudaEventDestroy(s->params_ready);
    for (auto st : s->streams)
      if (st) cudaStreamDestroy(st);
  }
  delete s;
  return TFX_OK;
}

int tfx_session_set_chunk_bytes(tfx_session* s, int64_t bytes) {
  const char* op = "tfx_session";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(bytes >= 4096, op, "chunk_bytes", "must be at least 4096");
  s->chunk_bytes = bytes;
  return TFX_OK;
}

// ---- LayerNorm (d, cols) ---------------------------------------------------------

}  // extern "C"

template <typename T, class K>
static int session_layernorm(tfx_session* s, const char* op, const T* x, const T* w, const T* b,
                             T* y, int64_t d, int64_t cols, K kernel) {
  TFX_REQUIRE(d >= 0 && cols >= 0, op, "shape", "extents must be non-negative");
  if (d == 0 || cols == 0) return TFX_OK;
  TFX_REQUIRE(x && w && y, op, !x ? "x" : (!w ? "weight" : "y"), "null pointer");
  std::vector<const void*> dev;
  int rc = upload_params(s, op, {{w, size_t(d) * sizeof(T)}, {b, b ? size_t(d) * sizeof(T) : 0}},
                         &dev);
  if (rc != TFX_OK) return rc;
  const int64_t per = units_per_chunk(s, 2 * d * int64_t(sizeof(T)));
  rc = ensure_slots(s, size_t(2 * per * d) * sizeof(T), op);
  if (rc != TFX_OK) return rc;
  const T* wd = static_cast<const T*>(dev[0]);
  const T* bd = static_cast<const T*>(dev[1]);
  return pipeline(s, op, cols, per, [&](int64_t c0, int64_t n, cudaStream_t st, char* slot) {
    T* in = reinterpret_cast<T*>(slot);
    T* out = in + per * d;
    int r = h2d(op, in, x + c0 * d, size_t(n * d) * sizeof(T), st);
    if (r == TFX_OK) r = kernel(in, wd, bd, out, d, n, st);
    if (r == TFX_OK) r = d2h(op, y + c0 * d, out, size_t(n * d) * sizeof(T), st);
    return r;
  });
}

extern "C" {

int tfx_session_layernorm_ff_f32(tfx_session* s, const float* x, const float* weight,
                                 const float* bias, float* y, int64_t d, int64_t cols,
                                 float eps) {
  const char* op = "tenferro-ext::layernorm_ff";
  TFX_SESSION_ENTER(op);
  return session_layernorm<float>(
      s, op, x, weight, bias, y, d, cols,
      [&](const float* in, const float* w, const float* b, float* out, int64_t dd, int64_t n,
          cudaStream_t st) { return tfx_layernorm_ff_f32(in, w, b, out, dd, n, eps, st); });
}

int tfx_session_layernorm_ff_f64(tfx_session* s, const double* x, const double* weight,
                                 const double* bias, double* y, int64_t d, int64_t cols,
                                 double eps) {
  const char* op = "tenferro-infer::layer_norm";
  TFX_SESSION_ENTER(op);
  return session_layernorm<double>(
      s, op, x, weight, bias, y, d, cols,
      [&](const double* in, const double* w, const double* b, double* out, int64_t dd,
          int64_t n, cudaStream_t st) { return tfx_layernorm_ff_f64(in, w, b, out, dd, n, eps, st); });
}

// The residual add fused into the LayerNorm that follows it: a and b in, the
// sum (when sum_out is not NULL) and y out, per chunk of columns.
int tfx_session_add_layernorm_ff_f32(tfx_session* s, const float* a, const float* b,
                                     const float* weight, const float* bias, float* sum_out,
                                     float* y, int64_t d, int64_t cols, float eps) {
  const char* op = "tenferro-ext::add_layernorm_ff";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(d >= 0 && cols >= 0, op, "shape", "extents must be non-negative");
  if (d == 0 || cols == 0) return TFX_OK;
  TFX_REQUIRE(a && b && weight && y, op, !a ? "a" : (!b ? "b" : (!weight ? "weight" : "y")),
              "null pointer");
  std::vector<const void*> dev;
  int rc = upload_params(s, op, {{weight, size_t(d) * 4}, {bias, bias ? size_t(d) * 4 : 0}},
                         &dev);
  if (rc != TFX_OK) return rc;
  const int64_t planes = sum_out ? 4 : 3;  // a, b, y (+ sum)
  const int64_t per = units_per_chunk(s, planes * d * 4);
  rc = ensure_slots(s, size_t(planes * per * d) * 4, op);
  if (rc != TFX_OK) return rc;
  const float* wd = static_cast<const float*>(dev[0]);
  const float* bd = static_cast<const float*>(dev[1]);
  return pipeline(s, op, cols, per, [&](int64_t c0, int64_t n, cudaStream_t st, char* slot) {
    float* ia = reinterpret_cast<float*>(slot);
    float* ib = ia + per * d;
    float* oy = ib + per * d;
    float* os = sum_out ? oy + per * d : nullptr;
    const size_t bytes = size_t(n * d) * 4;
    int r = h2d(op, ia, a + c0 * d, bytes, st);
    if (r == TFX_OK) r = h2d(op, ib, b + c0 * d, bytes, st);
    if (r == TFX_OK) r = tfx_add_layernorm_ff_f32(ia, ib, wd, bd, os, oy, d, n, eps, st);
    if (r == TFX_OK && os) r = d2h(op, sum_out + c0 * d, os, bytes, st);
    if (r == TFX_OK) r = d2h(op, y + c0 * d, oy, bytes, st);
    return r;
  });
}

// ---- RMSNorm (rows, width), feature-last: chunks of rows are strided blocks ------

int tfx_session_rmsnorm_last_f32(tfx_session* s, const float* x, const float* weight, float* y,
                                 int64_t rows, int64_t width, int centered, float eps) {
  const char* op = "tenferro-ext::rms_norm_last";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(rows >= 0 && width >= 0, op, "shape", "extents must be non-negative");
  if (rows == 0 || width == 0) return TFX_OK;
  TFX_REQUIRE(x && weight && y, op, !x ? "x" : (!weight ? "weight" : "y"), "null pointer");
  std::vector<const void*> dev;
  int rc = upload_params(s, op, {{weight, size_t(width) * 4}}, &dev);
  if (rc != TFX_OK) return rc;
  const int64_t per = units_per_chunk(s, 2 * width * 4, 4);
  rc = ensure_slots(s, size_t(2 * per * width) * 4, op);
  if (rc != TFX_OK) return rc;
  const float* wd = static_cast<const float*>(dev[0]);
  return pipeline(s, op, rows, per, [&](int64_t r0, int64_t n, cudaStream_t st, char* slot) {
    float* in = reinterpret_cast<float*>(slot);
    float* out = in + per * width;
    cudaError_t err = cudaMemcpy2DAsync(in, size_t(n) * 4, x + r0, size_t(rows) * 4,
                                        size_t(n) * 4, size_t(width), cudaMemcpyHostToDevice, st);
    if (err != cudaSuccess) return cuda_fail(op, "copy to device", err);
    int r = tfx_rmsnorm_last_f32(in, wd, out, n, width, centered, eps, st);
    if (r != TFX_OK) return r;
    err = cudaMemcpy2DAsync(y + r0, size_t(rows) * 4, out, size_t(n) * 4, size_t(n) * 4,
                            size_t(width), cudaMemcpyDeviceToHost, st);
    return err == cudaSuccess ? TFX_OK : cuda_fail(op, "copy to host", err);
  }, 4);
}

// ---- elementwise -----------------------------------------------------------------

}  // extern "C"

template <class K>
static int session_unary(tfx_session* s, const char* op, const float* x, float* y, int64_t n,
                         K kernel) {
  TFX_REQUIRE(n >= 0, op, "n", "must be non-negative");
  if (n == 0) return TFX_OK;
  TFX_REQUIRE(x && y, op, x ? "y" : "x", "null pointer");
  const int64_t per = units_per_chunk(s, 8, 64);
  int rc = ensure_slots(s, size_t(2 * per) * 4, op);
  if (rc != TFX_OK) return rc;
  return pipeline(s, op, n, per, [&](int64_t i0, int64_t m, cudaStream_t st, char* slot) {
    float* in = reinterpret_cast<float*>(slot);
    float* out = in + per;
    int r = h2d(op, in, x + i0, size_t(m) * 4, st);
    if (r == TFX_OK) r = kernel(in, out, m, st);
    if (r == TFX_OK) r = d2h(op, y + i0, out, size_t(m) * 4, st);
    return r;
  }, 64);
}

extern "C" {

int tfx_session_erf_f32(tfx_session* s, const float* x, float* y, int64_t n) {
  const char* op = "tenferro-ext::erf";
  TFX_SESSION_ENTER(op);
  return session_unary(s, op, x, y, n, [](const float* a, float* b, int64_t m, cudaStream_t st) {
    return tfx_erf_f32(a, b, m, st);
  });
}

int tfx_session_gelu_erf_f32(tfx_session* s, const float* x, float* y, int64_t n) {
  const char* op = "tenferro-ext::gelu_erf";
  TFX_SESSION_ENTER(op);
  return session_unary(s, op, x, y, n, [](const float* a, float* b, int64_t m, cudaStream_t st) {
    return tfx_gelu_erf_f32(a, b, m, st);
  });
}

}  // extern "C"

template <class K>
static int session_binary(tfx_session* s, const char* op, const float* a, const float* b,
                          float* y, int64_t n, K kernel) {
  TFX_REQUIRE(n >= 0, op, "n", "must be non-negative");
  if (n == 0) return TFX_OK;
  TFX_REQUIRE(a && b && y, op, !a ? "a" : (!b ? "b" : "y"), "null pointer");
  const int64_t per = units_per_chunk(s, 12, 64);
  int rc = ensure_slots(s, size_t(3 * per) * 4, op);
  if (rc != TFX_OK) return rc;
  return pipeline(s, op, n, per, [&](int64_t i0, int64_t m, cudaStream_t st, char* slot) {
    float* ia = reinterpret_cast<float*>(slot);
    float* ib = ia + per;
    float* out = ib + per;
    int r = h2d(op, ia, a + i0, size_t(m) * 4, st);
    if (r == TFX_OK) r = h2d(op, ib, b + i0, size_t(m) * 4, st);
    if (r == TFX_OK) r = kernel(ia, ib, out, m, st);
    if (r == TFX_OK) r = d2h(op, y + i0, out, size_t(m) * 4, st);
    return r;
  }, 64);
}

extern "C" {

int tfx_session_gated_silu_f32(tfx_session* s, const float* gate, const float* up, float* y,
                               int64_t n) {
  const char* op = "tenferro-ext::gated_silu";
  TFX_SESSION_ENTER(op);
  return session_binary(s, op, gate, up, y, n,
                        [](const float* g, const float* u, float* o, int64_t m, cudaStream_t st) {
                          return tfx_gated_silu_f32(g, u, o, m, st);
                        });
}

int tfx_session_add_f32(tfx_session* s, const float* a, const float* b, float* y, int64_t n) {
  const char* op = "tenferro-ext::add";
  TFX_SESSION_ENTER(op);
  return session_binary(s, op, a, b, y, n,
                        [](const float* p, const float* q, float* o, int64_t m, cudaStream_t st) {
                          return tfx_add_f32(p, q, o, m, st);
                        });
}

int tfx_session_geglu_ff_f32(tfx_session* s, const float* u, float* y, int64_t inter,
                             int64_t cols) {
  const char* op = "tenferro-ext::geglu";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(inter >= 0 && cols >= 0, op, "shape", "extents must be non-negative");
  if (inter == 0 || cols == 0) return TFX_OK;
  TFX_REQUIRE(u && y, op, u ? "y" : "u", "null pointer");
  const int64_t per = units_per_chunk(s, 3 * inter * 4);
  int rc = ensure_slots(s, size_t(3 * per * inter) * 4, op);
  if (rc != TFX_OK) return rc;
  return pipeline(s, op, cols, per, [&](int64_t c0, int64_t n, cudaStream_t st, char* slot) {
    float* in = reinterpret_cast<float*>(slot);
    float* out = in + 2 * per * inter;
    int r = h2d(op, in, u + c0 * 2 * inter, size_t(2 * n * inter) * 4, st);
    if (r == TFX_OK) r = tfx_geglu_ff_f32(in, out, inter, n, st);
    if (r == TFX_OK) r = d2h(op, y + c0 * inter, out, size_t(n * inter) * 4, st);
    return r;
  });
}

int tfx_session_bias_act_ff_f32(tfx_session* s, const float* x, const float* bias, float* y,
                                int64_t features, int64_t tokens, int act) {
  const char* op = "tenferro-ext::gemm_bias";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(features >= 0 && tokens >= 0, op, "shape", "extents must be non-negative");
  if (features == 0 || tokens == 0) return TFX_OK;
  TFX_REQUIRE(x && y, op, x ? "y" : "x", "null pointer");
  std::vector<const void*> dev;
  int rc = upload_params(s, op, {{bias, bias ? size_t(features) * 4 : 0}}, &dev);
  if (rc != TFX_OK) return rc;
  const int64_t per = units_per_chunk(s, 2 * features * 4);
  rc = ensure_slots(s, size_t(2 * per * features) * 4, op);
  if (rc != TFX_OK) return rc;
  const float* bd = static_cast<const float*>(dev[0]);
  return pipeline(s, op, tokens, per, [&](int64_t t0, int64_t n, cudaStream_t st, char* slot) {
    float* in = reinterpret_cast<float*>(slot);
    float* out = in + per * features;
    int r = h2d(op, in, x + t0 * features, size_t(n * features) * 4, st);
    if (r == TFX_OK) r = tfx_bias_act_ff_f32(in, bd, out, features, n, act, st);
    if (r == TFX_OK) r = d2h(op, y + t0 * features, out, size_t(n * features) * 4, st);
    return r;
  });
}

}  // extern "C"

// ---- GEMM with a fused epilogue: weight and bias uploaded once, token chunks ------
//
// x chunks (in_dim x n) in, y chunks (nout x n) out; chunks are whole
// 128-token tiles of the tensor-core kernel where the call allows.
template <class Launch>
static int session_gemm(tfx_session* s, const char* op, const float* x, const float* weight,
                        const float* bias, float* y, int64_t in_dim, int64_t nproj,
                        int64_t nout, int64_t length, Launch launch) {
  TFX_REQUIRE(in_dim >= 0 && nproj >= 0 && nout >= 0 && length >= 0, op, "shape",
              "extents must be non-negative");
  if (nout == 0 || length == 0) return TFX_OK;
  TFX_REQUIRE(x || in_dim == 0, op, "x", "null pointer");
  TFX_REQUIRE(weight || in_dim == 0, op, "weight", "null pointer");
  TFX_REQUIRE(y, op, "y", "null pointer");
  std::vector<const void*> dev;
  int rc = upload_params(s, op, {{weight, size_t(in_dim) * size_t(nproj) * 4},
                                 {bias, bias ? size_t(nproj) * 4 : 0}},
                         &dev);
  if (rc != TFX_OK) return rc;
  const int64_t per = units_per_chunk(s, (in_dim + nout) * 4, 128);
  rc = ensure_slots(s, size_t(per * (in_dim + nout)) * 4, op);
  if (rc != TFX_OK) return rc;
  const float* wd = static_cast<const float*>(dev[0]);
  const float* bd = static_cast<const float*>(dev[1]);
  return pipeline(
      s, op, length, per,
      [&](int64_t t0, int64_t n, cudaStream_t st, char* slot) {
        float* in = reinterpret_cast<float*>(slot);
        float* out = in + per * in_dim;
        int r = in_dim ? h2d(op, in, x + t0 * in_dim, size_t(n * in_dim) * 4, st) : TFX_OK;
        if (r == TFX_OK) r = launch(in, wd, bd, out, n, st);
        if (r == TFX_OK) r = d2h(op, y + t0 * nout, out, size_t(n * nout) * 4, st);
        return r;
      },
      128);
}

extern "C" {

int tfx_session_gemm_geglu_ff_f32(tfx_session* s, const float* x, const float* weight,
                                  const float* bias, float* y, int64_t in_dim,
                                  int64_t intermediate, int64_t length) {
  const char* op = "tenferro-ext::gemm_geglu";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(intermediate < (int64_t(1) << 29), op, "intermediate",
              "projected feature extent overflow");
  return session_gemm(s, op, x, weight, bias, y, in_dim, 2 * intermediate, intermediate, length,
                      [&](const float* xi, const float* w, const float* b, float* yo, int64_t n,
                          cudaStream_t st) {
                        return tfx_gemm_geglu_ff_f32(xi, w, b, yo, in_dim, intermediate, n, st);
                      });
}

int tfx_session_gemm_bias_act_ff_f32(tfx_session* s, const float* x, const float* weight,
                                     const float* bias, float* y, int64_t in_dim, int64_t out_dim,
                                     int64_t length, int act) {
  const char* op = "tenferro-ext::gemm_bias";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(act == TFX_ACT_IDENTITY || act == TFX_ACT_GELU_ERF || act == TFX_ACT_RELU, op,
              "act", "unknown activation " + std::to_string(act));
  return session_gemm(s, op, x, weight, bias, y, in_dim, out_dim, out_dim, length,
                      [&](const float* xi, const float* w, const float* b, float* yo, int64_t n,
                          cudaStream_t st) {
                        return tfx_gemm_bias_act_ff_f32(xi, w, b, yo, in_dim, out_dim, n, act,
                                                        st);
                      });
}

// ---- masked softmax: chunks of whole rows; mask tensors uploaded once ------------

static int64_t extent(int64_t n0, int64_t s0, int64_t n1, int64_t s1, int64_t n2, int64_t s2) {
  return 1 + (n0 - 1) * s0 + (n1 - 1) * s1 + (n2 - 1) * s2;
}

int tfx_session_masked_softmax_f32(tfx_session* s, const float* scores, float* probs,
                                   const tfx_softmax_desc* desc) {
  const char* op = "tenferro-infer::masked_softmax";
  TFX_SESSION_ENTER(op);
  int64_t rows = 0;
  int rc = validate_softmax(scores, probs, desc, &rows);
  if (rc != TFX_OK || rows == 0) return rc;
  tfx_softmax_desc d = *desc;
  TFX_REQUIRE(d.add_stride_b >= 0 && d.add_stride_q >= 0 && d.add_stride_k >= 0 &&
                  d.keep_stride_b >= 0 && d.keep_stride_q >= 0 && d.keep_stride_k >= 0,
              op, "mask", "mask strides must be non-negative");
  const size_t vl_bytes = d.valid_lens ? size_t(d.batch) * 4 : 0;
  const size_t add_bytes =
      d.add_mask ? size_t(extent(d.batch, d.add_stride_b, d.q_len, d.add_stride_q, d.k_len,
                                 d.add_stride_k)) * 4 : 0;
  const size_t keep_bytes =
      d.keep ? size_t(extent(d.batch, d.keep_stride_b, d.q_len, d.keep_stride_q, d.k_len,
                             d.keep_stride_k)) : 0;
  std::vector<const void*> dev;
  rc = upload_params(s, op, {{d.valid_lens, vl_bytes}, {d.add_mask, add_bytes}, {d.keep, keep_bytes}},
                     &dev);
  if (rc != TFX_OK) return rc;
  d.valid_lens = static_cast<const int32_t*>(dev[0]);
  d.add_mask = static_cast<const float*>(dev[1]);
  d.keep = static_cast<const uint8_t*>(dev[2]);
  const int64_t L = d.k_len;
  const int64_t per = units_per_chunk(s, 2 * L * 4);
  rc = ensure_slots(s, size_t(2 * per * L) * 4, op);
  if (rc != TFX_OK) return rc;
  return pipeline(s, op, rows, per, [&](int64_t r0, int64_t n, cudaStream_t st, char* slot) {
    float* in = reinterpret_cast<float*>(slot);
    float* out = in + per * L;
    int r = h2d(op, in, scores + r0 * L, size_t(n * L) * 4, st);
    if (r == TFX_OK) r = masked_softmax_rows(in, out, &d, r0, n, st);
    if (r == TFX_OK) r = d2h(op, probs + r0 * L, out, size_t(n * L) * 4, st);
    return r;
  });
}

// ---- RoPE: y is x with the described vectors rotated --------------------------------

int tfx_session_rope_pairhalf_f32(tfx_session* s, const float* x, float* y, double base,
                                  const tfx_rope_desc* desc) {
  const char* op = "tenferro-infer::rope";
  TFX_SESSION_ENTER(op);
  TFX_REQUIRE(desc, op, "desc", "null pointer");
  const tfx_rope_desc d = *desc;
  TFX_REQUIRE(d.n_vec >= 0 && d.seq >= 0 && d.batch >= 0 && d.head_dim >= 0, op, "shape",
              "extents must be non-negative");
  TFX_REQUIRE(d.rotary_dim > 0 && d.rotary_dim % 2 == 0 && d.rotary_dim <= d.head_dim, op,
              "rotary_dim", "must be positive, even and at most head_dim");
  if (d.n_vec == 0 || d.seq == 0 || d.batch == 0) return TFX_OK;
  TFX_REQUIRE(x && y, op, x ? "y" : "x", "null pointer");
  TFX_REQUIRE(d.stride_vec >= 0 && d.stride_pos >= 0 && d.stride_batch >= 0 && d.stride_feat > 0,
              op, "strides", "strides must be non-negative (stride_feat positive)");
  auto key = std::make_tuple(base, d.seq, d.rotary_dim);
  auto it = s->tables.find(key);
  if (it == s->tables.end()) {
    const size_t n = size_t(d.seq * (d.rotary_dim / 2));
    std::vector<float> c(n), sn(n);
    int rc = tfx_rope_tables_f32(base, d.seq, d.rotary_dim, c.data(), sn.data());
    if (rc != TFX_OK) return rc;
    if (s->tables.size() > 16) s->tables.clear();
    it = s->tables.emplace(key, std::make_pair(std::move(c), std::move(sn))).first;
  }
  std::vector<const void*> dev;
  int rc = upload_params(s, op, {{it->second.first.data(), it->second.first.size() * 4},
                                 {it->second.second.data(), it->second.second.size() * 4}},
                         &dev);
  if (rc != TFX_OK) return rc;
  const float* cd = static_cast<const float*>(dev[0]);
  const float* sd = static_cast<const float*>(dev[1]);
  // Common layout (a qkv tensor, or q / k alone): the vectors of one position
  // span W contiguous-channel floats at the start of a row, and rows (batch
  // item, position) are evenly pitched. Then only those W floats of each row
  // cross PCIe, as 2-D copies into a compact staging layout -- for the
  // feature-first qkv of the chain, q and k but not v.
  const int64_t W = (d.n_vec - 1) * d.stride_vec + (d.head_dim - 1) * d.stride_feat + 1;
  const int64_t pitch = d.seq > 1 ? d.stride_pos : (d.batch > 1 ? d.stride_batch : W);
  const bool rows2d = d.stride_feat == 1 && pitch >= W &&
                      (d.seq == 1 || d.batch == 1 || d.stride_batch == d.seq * d.stride_pos);
  if (rows2d) {
    const int64_t per2 = units_per_chunk(s, 2 * d.seq * W * 4);
    rc = ensure_slots(s, size_t(per2 * d.seq * W) * 4, op);
    if (rc != TFX_OK) return rc;
    return pipeline(s, op, d.batch, per2, [&](int64_t b0, int64_t n, cudaStream_t st, char* slot) {
      float* buf = reinterpret_cast<float*>(slot);
      const int64_t row0 = b0 * d.seq;
      cudaError_t err = cudaMemcpy2DAsync(buf, size_t(W) * 4, x + row0 * pitch, size_t(pitch) * 4,
                                          size_t(W) * 4, size_t(n * d.seq),
                                          cudaMemcpyHostToDevice, st);
      if (err != cudaSuccess) return cuda_fail(op, "copy to device", err);
      tfx_rope_desc cd_desc = d;
      cd_desc.batch = n;
      cd_desc.stride_pos = W;
      cd_desc.stride_batch = d.seq * W;
      const int r = tfx_rope_pairhalf_f32(buf, buf, cd, sd, &cd_desc, st);
      if (r != TFX_OK) return r;
      err = cudaMemcpy2DAsync(y + row0 * pitch, size_t(pitch) * 4, buf, size_t(W) * 4,
                              size_t(W) * 4, size_t(n * d.seq), cudaMemcpyDeviceToHost, st);
      return err == cudaSuccess ? TFX_OK : cuda_fail(op, "copy to host", err);
    });
  }
  // Extent of one batch item; batch items are chunked when they are laid out
  // one after another (batch is the outermost axis).
  const int64_t item = 1 + (d.n_vec - 1) * d.stride_vec + (d.seq - 1) * d.stride_pos +
                       (d.head_dim - 1) * d.stride_feat;
  const bool batch_outer = d.batch == 1 || d.stride_batch >= item;
  const int64_t unit = batch_outer ? (d.batch == 1 ? item : d.stride_batch) : 0;
  const int64_t total = batch_outer ? (d.batch - 1) * unit + item
                                    : item + (d.batch - 1) * d.stride_batch;
  const int64_t per = batch_outer ? units_per_chunk(s, 2 * unit * 4) : d.batch;
  const int64_t span = batch_outer ? (per - 1) * unit + item : total;
  rc = ensure_slots(s, size_t(span) * 4, op);
  if (rc != TFX_OK) return rc;
  return pipeline(s, op, d.batch, per, [&](int64_t b0, int64_t n, cudaStream_t st, char* slot) {
    float* buf = reinterpret_cast<float*>(slot);
    const int64_t first = batch_outer ? b0 * unit : 0;
    const int64_t len = batch_outer ? (n - 1) * unit + item : total;
    int r = h2d(op, buf, x + first, size_t(len) * 4, st);
    tfx_rope_desc cd_desc = d;
    cd_desc.batch = n;
    if (r == TFX_OK) r = tfx_rope_pairhalf_f32(buf, buf, cd, sd, &cd_desc, st);
    if (r == TFX_OK) r = d2h(op, y + first, buf, size_t(len) * 4, st);
    return r;
  });
}

}  // extern "C"
