// tma.cuh -- tensor-memory-accelerator (TMA) tile loads into shared memory,
// completed through mbarrier transaction counts, and bounded waits on them.
//
// A load is one cp.async.bulk.tensor of a box described by a CUtensorMap that
// the host encodes (cuTensorMapEncodeTiled, reached through the runtime's
// driver entry point so the library does not link libcuda). Every load here
// goes to the issuing CTA only, and every tensor map covers this GPU's own
// memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace tfx {

// Host: encodes a 2-D f32 tensor map over base[i0 + stride1 * i1] (i0 < dim0,
// i1 < dim1, stride1 in elements) with box (box0, box1), zero fill out of
// bounds, and no swizzle (swizzle_bytes 0) or the 64- / 128-byte swizzle of
// tc.cuh's operand layouts (swizzle_bytes == box0 * 4). Returns false and sets
// *why when the driver refuses.
bool encode_map_2d_f32(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                       uint64_t stride1, uint32_t box0, uint32_t box1, std::string* why,
                       int swizzle_bytes = 0);

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes initialised mbarriers visible to the async proxy (the TMA unit).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One arrival that also announces `bytes` of transactions for the phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// One plain arrival.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete; gives up (false)
// after `limit_cycles` SM clock cycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit_cycles) return false;
  }
  return true;
}

// Orders this thread's earlier generic-proxy accesses to shared memory before
// later async-proxy (TMA) accesses to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Box at coordinates (c0, c1) of `map` into shared memory at dst (128-byte
// aligned); completes `bytes of the box` transactions on bar. c0 * 4 bytes
// must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace tfx
