// common.cuh -- shared host/device helpers of libtfx: status reporting,
// per-device attributes, 128-bit streaming loads/stores, warp reductions and
// 32-bit fast division for index decomposition.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>

#include "tfx.h"

namespace tfx {

// ---- status ----------------------------------------------------------------

// Records "op: field: message" as this thread's last error and returns code.
int fail(int code, const char* op, const char* field, const std::string& message);
// Clears this thread's last error.
void clear_error();
// Checks the launch that was just enqueued; TFX_ERR_CUDA with the runtime's
// message if it failed.
int check_launch(const char* op);

// ---- per-device attributes ---------------------------------------------------

struct DeviceInfo {
  int device = -1;
  int sms = 0;
  int max_threads_per_sm = 0;
  int l2_bytes = 0;
  int smem_optin = 0;  // largest dynamic shared memory one CTA may opt in to
  int cc_major = 0, cc_minor = 0;
};
// The current device's attributes, read once per device.
const DeviceInfo& device_info(int* status);

// Stream-ordered scratch from a per-device memory pool owned by libtfx (the
// caller's default pool is left alone). The pool keeps up to 1 GiB of freed
// scratch mapped across synchronisations, so calls that need the same
// scratch again do not map fresh memory; free with cudaFreeAsync.
cudaError_t scratch_malloc(void** ptr, size_t bytes, cudaStream_t stream);

// ---- argument checks -----------------------------------------------------------

inline bool aligned(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

// True when [a, a+na) and [b, b+nb) (bytes) share any byte.
inline bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + nb && pb < pa + na;
}

// ---- device helpers --------------------------------------------------------

// Read-only, not-retained-in-L1 loads for data streamed once. Every kernel
// here reads each input address once, before the same thread writes that
// address (in-place calls), so the non-coherent path never sees a value the
// kernel itself has written.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float2 ld_stream(const float2* p) {
  float2 v;
  asm("ld.global.nc.L1::no_allocate.v2.f32 {%0, %1}, [%2];"
               : "=f"(v.x), "=f"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_stream(const float* p) {
  float v;
  asm("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ double2 ld_stream(const double2* p) {
  double2 v;
  asm("ld.global.nc.L1::no_allocate.v2.f64 {%0, %1}, [%2];"
               : "=d"(v.x), "=d"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ double ld_stream(const double* p) {
  double v;
  asm("ld.global.nc.L1::no_allocate.f64 %0, [%1];" : "=d"(v) : "l"(p));
  return v;
}

// Programmatic dependent launch. Every kernel here is launched with
// programmatic stream serialisation (launch_kernel below), so it may start
// while the previous kernel on the stream is still finishing. It must call
// pdl_wait() before touching global memory: that returns once the previous
// grid has completed and its writes are visible (and guards against
// overwriting what the previous grid still reads).
//
// Kernels do not trigger their dependents early (pdl_launch_dependents at the
// start): the next grid's CTAs would then take the SM slots that free up first
// and pile onto those SMs while the current grid still runs, and a grid whose
// CTAs each own a fixed share of the work (one wave, or a persistent grid) is
// then only as fast as its most loaded SM. Measured on configs[0] LayerNorm
// (one wave of 1024 CTAs): 10.46 us with the early trigger, 9.88 us without;
// the whole configs[4] chain 0.4502 -> 0.4437 ms per step, and 0.4516 with no
// programmatic launch at all. Without the early trigger the next grid is
// launched as the last CTAs of this one exit, before its completion is
// signalled, which still hides most of the launch latency.
// TFX_PDL_EARLY_TRIGGER=1 at build time restores the early trigger.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#ifndef TFX_PDL_EARLY_TRIGGER
#define TFX_PDL_EARLY_TRIGGER 0
#endif
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
#if TFX_PDL_EARLY_TRIGGER
  pdl_launch_dependents();
#endif
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// q = n / d for 32-bit unsigned n and a runtime-constant divisor d >= 1
// (round-up multiplier, Granlund & Montgomery 1994 / Hacker's Delight 10-9).
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t divisor) : d(divisor) {
    if (d == 1) return;
    uint32_t l = 0;
    while ((uint64_t(1) << l) < d) ++l;
    m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1);
    s = l;
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (d == 1) return n;
#ifdef __CUDA_ARCH__
    const uint32_t t = __umulhi(n, m);
#else
    const uint32_t t = uint32_t((uint64_t(n) * m) >> 32);
#endif
    return (t + ((n - t) >> 1)) >> (s - 1);
  }
};

// Launches kernel<<<grid, block, smem, stream>>>(args...) with programmatic
// stream serialisation allowed (see pdl_wait) and, when cluster > 1, a
// (cluster, 1, 1) thread-block cluster; then reports failures as check_launch
// does.
template <typename... KArgs, typename... Args>
int launch_kernel(const char* op, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                  cudaStream_t stream, unsigned cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
#ifndef TFX_PDL_ATTR
#define TFX_PDL_ATTR 1
#endif
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = TFX_PDL_ATTR;
  unsigned n = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(TFX_ERR_CUDA, op, "launch",
                std::string(cudaGetErrorName(err)) + ": " + cudaGetErrorString(err));
  }
  return check_launch(op);
}

}  // namespace tfx

// Validation helpers shared by the entry points.
#define TFX_REQUIRE(cond, op, field, msg)                                   \
  do {                                                                      \
    if (!(cond)) return ::tfx::fail(TFX_ERR_INVALID_ARGUMENT, op, field, msg); \
  } while (0)
