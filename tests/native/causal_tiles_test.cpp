// Host check of causal_tiles.cuh, the work enumeration of the batched
// tensor-core GEMM on a causal square contraction (compiled with g++: the
// CUDA qualifiers are defined away).
//
//  * live_row / live_prefix: live score tile r of a batch maps to the tile row
//    whose range holds it, and the rows' live tiles are exactly n <= lm / 2
//    (256-key output tiles at or below a 128-query tile's diagonal);
//  * CausalKSplit: walking every CTA's contiguous run of 128-key chunks the
//    way the GEMM does covers each chunk once; the pieces of a tile carry
//    slots 0, 1, ... in order, their count is pieces(), their stages add up
//    to the tile's contraction, and max_pieces() bounds them all.
// Prints "bad=0" when every check holds.
#define __host__
#define __device__
#define __forceinline__ inline
#include <algorithm>
#include <cstdio>
#include <map>
#include <utility>
#include <vector>

#include "causal_tiles.cuh"

using namespace tfx;

int main() {
  long bad = 0;
  for (uint64_t r = 0; r < 2000000; ++r) {
    const uint32_t lm = live_row(r);
    if (!(live_prefix(lm) <= r && r < live_prefix(lm + 1))) ++bad;
    const uint32_t l2 = CausalKSplit::row_of(r);
    if (!(CausalKSplit::prefix(l2) <= r && r < CausalKSplit::prefix(l2 + 1))) ++bad;
  }
  for (uint32_t lm = 0; lm < 512; ++lm)  // live tiles of row lm: n * 256 <= 128 lm + 127
    if (live_prefix(lm + 1) - live_prefix(lm) != (128 * lm + 127) / 256 + 1) ++bad;

  int cases = 0;
  // cs: 32-key stages per chunk -- 4 (128-token rows, one CTA per tile) or 8
  // (256-token pair rows on CTA pairs)
  for (uint32_t cs : {4u, 8u})
  for (uint32_t batches : {1u, 2u, 3u, 8u, 16u, 64u})
    for (uint32_t mb : {1u, 2u, 3u, 5u, 16u, 33u, 64u})
      for (uint32_t sms : {1u, 7u, 74u, 148u, 1000u}) {
        const CausalKSplit sp = causal_k_split(batches, mb, sms, 32 * cs);
        if (sp.row_tokens != 32 * cs) ++bad;
        const uint32_t nst = cs * mb;  // 32-key stages of a batch's contraction
        std::map<std::pair<uint32_t, uint32_t>, std::vector<std::pair<uint32_t, uint32_t>>> tiles;
        std::vector<int> covered(sp.items, 0);
        for (uint32_t b = 0; b < sp.grid; ++b) {
          uint64_t i = sp.start(b);
          const uint64_t end = sp.start(b + 1);
          while (i < end) {  // the GEMM's next_piece for kCausalK
            const uint32_t batch = uint32_t(i / sp.per_batch);
            const uint64_t r = i - uint64_t(batch) * sp.per_batch;
            const uint32_t lm = CausalKSplit::row_of(r);
            const uint32_t c0 = uint32_t(r - CausalKSplit::prefix(lm));
            const uint32_t c1 =
                uint32_t(std::min<uint64_t>(uint64_t(lm) + 1, uint64_t(c0) + (end - i)));
            const uint32_t slot = b - sp.owner(sp.first(batch, lm));
            const uint32_t s0 = c0 * cs, s1 = std::min(nst, c1 * cs);
            if (s1 <= s0) ++bad;
            for (uint64_t k = i; k < i + (c1 - c0); ++k) covered[k]++;
            tiles[{batch, lm}].push_back({slot, s1 - s0});
            i += c1 - c0;
          }
        }
        for (int c : covered)
          if (c != 1) ++bad;
        const uint32_t maxp = sp.max_pieces(batches);
        for (const auto& kv : tiles) {
          const uint32_t want = sp.pieces(kv.first.first, kv.first.second);
          if (kv.second.size() != want || want > maxp) ++bad;
          uint32_t stages = 0;
          for (uint32_t p = 0; p < kv.second.size(); ++p) {
            if (kv.second[p].first != p) ++bad;
            stages += kv.second[p].second;
          }
          if (stages != cs * (kv.first.second + 1)) ++bad;
        }
        if (tiles.size() != size_t(batches) * mb) ++bad;
        ++cases;
      }
  std::printf("cases=%d bad=%ld\n", cases, bad);
  return bad == 0 ? 0 : 1;
}
