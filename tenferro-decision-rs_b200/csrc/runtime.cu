// runtime.cu -- status reporting and per-device attribute cache of libtfx,
// plus the host-only helpers of tfx.h.

#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace tfx {

namespace {
thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::once_flag g_once[kMaxDevices];
int g_status[kMaxDevices];
}  // namespace

int fail(int code, const char* op, const char* field, const std::string& message) {
  g_last_error = std::string(op) + ": " + field + ": " + message;
  return code;
}

void clear_error() { g_last_error.clear(); }

int check_launch(const char* op) {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess)
    return fail(TFX_ERR_CUDA, op, "launch", std::string(cudaGetErrorName(err)) + ": " +
                                                cudaGetErrorString(err));
  return TFX_OK;
}

const DeviceInfo& device_info(int* status) {
  static DeviceInfo invalid;
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = fail(TFX_ERR_CUDA, "tfx", "device",
                   err != cudaSuccess ? cudaGetErrorString(err) : "device ordinal out of range");
    return invalid;
  }
  std::call_once(g_once[dev], [dev] {
    DeviceInfo& d = g_info[dev];
    d.device = dev;
    g_status[dev] = TFX_OK;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_threads_per_sm, cudaDevAttrMaxThreadsPerMultiProcessor,
                               dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) !=
            cudaSuccess) {
      g_status[dev] = TFX_ERR_CUDA;
    }
  });
  if (g_status[dev] != TFX_OK) {
    *status = fail(TFX_ERR_CUDA, "tfx", "device", "cannot read device attributes");
    return invalid;
  }
  if (g_info[dev].cc_major != 10) {
    *status = fail(TFX_ERR_UNSUPPORTED, "tfx", "device",
                   "libtfx is built for sm_100a (B200); device " + std::to_string(dev) +
                       " is sm_" + std::to_string(g_info[dev].cc_major) +
                       std::to_string(g_info[dev].cc_minor));
    return invalid;
  }
  *status = TFX_OK;
  return g_info[dev];
}

namespace {
cudaMemPool_t g_pool[kMaxDevices];
std::once_flag g_pool_once[kMaxDevices];
}  // namespace

cudaError_t scratch_malloc(void** ptr, size_t bytes, cudaStream_t stream) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaMallocAsync(ptr, bytes, stream);
  std::call_once(g_pool_once[dev], [dev] {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      cudaGetLastError();
      return;  // scratch then comes from the device's default pool
    }
    uint64_t keep = uint64_t(1) << 30;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    g_pool[dev] = pool;
  });
  if (g_pool[dev] == nullptr) return cudaMallocAsync(ptr, bytes, stream);
  return cudaMallocFromPoolAsync(ptr, bytes, g_pool[dev], stream);
}

}  // namespace tfx

extern "C" {

const char* tfx_last_error_string(void) { return tfx::g_last_error.c_str(); }

int tfx_version(void) { return 10000; }

void tfx_softmax_desc_init(tfx_softmax_desc* desc, int64_t batch, int64_t heads, int64_t q_len,
                           int64_t k_len) {
  if (!desc) return;
  *desc = tfx_softmax_desc{};
  desc->batch = batch;
  desc->heads = heads;
  desc->q_len = q_len;
  desc->k_len = k_len;
  desc->scale = 1.0f;
  desc->semantics = TFX_SOFTMAX_EXCLUDE;
  desc->window = -1;
  desc->valid_len = -1;
}

// crates/tenferro-infer/src/rope.rs:84-92 (angle in f64) and table() :15-24
// (cos/sin rounded to f32); row-major (seq, rotary_dim/2).
int tfx_rope_tables_f32(double base, int64_t seq, int64_t rotary_dim, float* cos_host,
                        float* sin_host) {
  tfx::clear_error();
  const char* op = "tenferro-infer::rope";
  TFX_REQUIRE(seq >= 0, op, "seq", "must be non-negative");
  TFX_REQUIRE(rotary_dim > 0 && rotary_dim % 2 == 0, op, "rotary_dim",
              "rotary width must be a positive even number, got " + std::to_string(rotary_dim));
  TFX_REQUIRE(seq == 0 || (cos_host && sin_host), op, "tables", "null pointer");
  const int64_t half = rotary_dim / 2;
  for (int64_t p = 0; p < seq; ++p)
    for (int64_t i = 0; i < half; ++i) {
      const double theta = double(p) * std::pow(base, -2.0 * double(i) / double(rotary_dim));
      cos_host[p * half + i] = float(std::cos(theta));
      sin_host[p * half + i] = float(std::sin(theta));
    }
  return TFX_OK;
}

}  // extern "C"
