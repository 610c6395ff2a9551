// causal_tiles.cuh -- work enumeration of the batched tensor-core GEMM for a
// causal square contraction (per batch of T tokens, 128-token tiles lm = 0 ..
// mb - 1, T = 128 mb), shared by the GEMM and the kernels that consume its
// output.
//
//  * Scores (S = Q K^T, causal on the outputs): tile lm needs the 256-output
//    tiles n <= lm / 2 only. Live tiles are numbered batch by batch, lm by lm;
//    tile lm starts at live_prefix(lm).
//  * P V (causal on the contraction): tile lm contracts over keys < 128 (lm +
//    1), i.e. lm + 1 chunks of 128 keys. On CTA pairs the rows are 256 tokens
//    and the chunks 256 keys, with the same triangle. The chunks of all tiles, numbered
//    batch by batch, lm by lm, are split into contiguous runs, one per CTA
//    (CTA b owns chunks [start(b), start(b + 1))), so every CTA gets the same
//    amount of MMA work whatever the tile lengths. A tile whose chunks span
//    several CTAs is computed in pieces; piece p (the p-th CTA that holds some
//    of the tile's chunks) writes its own output slot p, and the consumer adds
//    the slots 0, 1, ... in that order (deterministic).
#pragma once

#include <cmath>
#include <cstdint>

namespace tfx {

// Live score tiles of rows [0, lm): sum over j < lm of (j / 2 + 1).
__host__ __device__ __forceinline__ uint64_t live_prefix(uint32_t lm) {
  const uint64_t p = lm / 2;
  return (lm & 1) ? (p + 1) * (p + 1) : p * (p + 1);
}

// The tile row holding live tile r of a batch.
__host__ __device__ __forceinline__ uint32_t live_row(uint64_t r) {
  uint32_t lm = uint32_t(2.0f * sqrtf(float(r)));
  while (lm > 0 && live_prefix(lm) > r) --lm;
  while (live_prefix(lm + 1) <= r) ++lm;
  return lm;
}

struct CausalKSplit {
  uint32_t mb;         // token tiles per batch (rows of the triangle)
  uint32_t row_tokens; // tokens per tile row and keys per chunk: 128, or 256 on CTA pairs
  uint32_t grid;       // CTAs
  uint64_t per_batch;  // chunks per batch: mb (mb + 1) / 2
  uint64_t items;      // chunks in all

  __host__ __device__ static uint64_t prefix(uint32_t lm) { return uint64_t(lm) * (lm + 1) / 2; }
  // The tile row holding chunk r of a batch.
  __host__ __device__ static uint32_t row_of(uint64_t r) {
    uint32_t lm = uint32_t((sqrtf(8.0f * float(r) + 1.0f) - 1.0f) * 0.5f);
    while (lm > 0 && prefix(lm) > r) --lm;
    while (prefix(lm + 1) <= r) ++lm;
    return lm;
  }
  __host__ __device__ uint64_t start(uint32_t b) const { return uint64_t(b) * items / grid; }
  // The CTA whose run holds chunk i: the largest b with start(b) <= i.
  __host__ __device__ uint32_t owner(uint64_t i) const {
    if (items * grid < (uint64_t(1) << 32))  // the usual case: 32-bit division
      return (uint32_t(i + 1) * grid - 1) / uint32_t(items);
    return uint32_t(((i + 1) * grid - 1) / items);
  }
  __host__ __device__ uint64_t first(uint32_t batch, uint32_t lm) const {
    return uint64_t(batch) * per_batch + prefix(lm);
  }
  // Output slots written for tile (batch, lm).
  __host__ __device__ uint32_t pieces(uint32_t batch, uint32_t lm) const {
    const uint64_t f = first(batch, lm);
    return owner(f + lm) - owner(f) + 1;
  }
  // The most slots any tile needs (host).
  uint32_t max_pieces(uint32_t batches) const {
    uint32_t m = 1;
    for (uint32_t b = 0; b < batches; ++b)
      for (uint32_t lm = 0; lm < mb; ++lm) {
        const uint32_t p = pieces(b, lm);
        m = p > m ? p : m;
      }
    return m;
  }
};

// The split for `batches` batches of mb tile rows of row_tokens tokens over
// at most `sms` CTAs (or CTA pairs).
inline CausalKSplit causal_k_split(uint32_t batches, uint32_t mb, uint32_t sms,
                                   uint32_t row_tokens = 128) {
  CausalKSplit s;
  s.mb = mb;
  s.row_tokens = row_tokens;
  s.per_batch = uint64_t(mb) * (mb + 1) / 2;
  s.items = s.per_batch * batches;
  s.grid = uint32_t(s.items < sms ? s.items : sms);
  return s;
}

}  // namespace tfx
