// tc.cuh -- fifth-generation tensor core (tcgen05) helpers for sm_100a:
// tensor-memory (TMEM) allocation, MMA issue with shared-memory descriptors,
// completion through mbarriers, and TMEM <-> register moves.
//
// Conventions used by the kernels here:
//   * operands in shared memory are "K-major, 128-byte swizzled": each row
//     (one M or N index) holds 32 f32/tf32 values of K in 128 bytes, the
//     16-byte chunks of row r permuted by chunk ^ (r % 8); 8 rows form a
//     1024-byte atom, atoms follow each other (stride 1024 bytes), and a
//     K range wider than 32 values continues in another such region.
//     This is the layout a TMA load with CU_TENSOR_MAP_SWIZZLE_128B and a
//     32-value inner box writes.
//   * an MMA of K = 8 tf32 values reads 32 bytes of every row: the
//     descriptor's start address moves by 32 bytes per K step inside a row
//     and to the next region every four steps.
//   * accumulators are f32 in TMEM: row m of the tile in lane m, column n of
//     the tile in column base + n.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "tma.cuh"

namespace tfx {

// Round a finite x to the nearest tf32 (10-bit mantissa, ties away from
// zero) on the integer pipe: adding half a tf32 ulp (bit 12) to the magnitude
// bits and clearing the 13 low bits -- the result cvt.rna.tf32.f32 gives for
// every finite x below the largest tf32, without the conversion unit (which
// the softmax's exponentials already load). The result is an f32 whose 13
// low mantissa bits are zero.
__device__ __forceinline__ float tf32_round_finite(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// Shared-memory matrix descriptor for a K-major SW128 operand starting at
// shared address `addr` (1024-byte atoms; +32 bytes per K step allowed).
// Fields: start >> 4 [0,14), leading byte offset 1 (unused for swizzled
// K-major) [16,30), stride byte offset 1024 >> 4 [32,46), version 1 [46,48),
// base offset 0, layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// The same for a K-major SW64 operand: rows of 64 bytes (16 f32 / tf32
// values of K), the 16-byte chunks of row r permuted by the 64-byte swizzle,
// 8-row atoms of 512 bytes (stride byte offset 512 >> 4), layout type
// SWIZZLE_64B = 4 [61,64). A K step of 8 tf32 values moves the start by 32
// bytes inside a row. This is the layout a TMA load with
// CU_TENSOR_MAP_SWIZZLE_64B and a 16-value inner box writes.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) | (uint64_t(512 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(4) << 61);
}

// Descriptor of an MN-major tf32 operand in the "128-byte swizzle, 32-byte
// atoms" layout, the only MN-major layout the tf32 MMA reads: 128-byte rows
// hold 32 consecutive values of N (M) for one K index, rows follow each other
// (128 bytes apart), and the four 32-byte granules of row r sit at granule
// index g ^ (r % 4) (address bits [5,7) XOR bits [7,9)). Groups of 4 rows are
// 512 bytes apart (stride byte offset); the next 32 values of N start
// `mn_stride` bytes further on (leading byte offset); layout type
// SWIZZLE_128B_BASE32B = 1 [61,64). A K step of 8 moves the start by 1024
// bytes.
__device__ __forceinline__ uint64_t smem_desc_sw128b32_mn(uint32_t addr, uint32_t mn_stride) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((mn_stride >> 4) & 0x3FFF) << 16) |
         (uint64_t(512 >> 4) << 32) | (uint64_t(1) << 46) | (uint64_t(1) << 61);
}

// Instruction descriptor of tcgen05.mma.kind::tf32, f32 accumulate, both
// operands K-major: c_format F32 [4,6), a/b_format TF32 [7,10) [10,13),
// N >> 3 [17,23), M >> 4 [24,29).
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// The same with B MN-major (transpose-B bit 16).
__host__ __device__ constexpr uint32_t idesc_tf32_bmn(int m, int n) {
  return idesc_tf32(m, n) | (1u << 16);
}

// D (+)= A * B^T with A and B in shared memory.
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// D (+)= A * B^T with A in TMEM (row m in lane m, K values in columns).
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrives once on `bar` when every tcgen05 operation this thread issued
// before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole warp: allocates `cols` TMEM columns (power of two >= 32) and writes
// the base address to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
// Whole warp.
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
               : "memory");
}

// 16 consecutive columns of this thread's lane (warp w of a warpgroup reads
// lanes 32w .. 32w+31; the address carries the lane in its upper half).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]),
      "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]),
      "f"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace tfx
