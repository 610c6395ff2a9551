// chunk_plan.h -- how a host-buffer session call splits its units (columns,
// rows, elements, batch items) into pipelined chunks. Host-only; shared by
// session.cu and the CPU test that checks its invariants.
#pragma once

#include <algorithm>
#include <cstdint>
#include <vector>

namespace tfx {

// Chunk sizes for `units` units with at most `per` per chunk. A call costs
// its copies plus the first chunk's copy-in (nothing else can run yet) and
// the last chunk's kernel and copy-out (nothing else is left to overlap), so
// the sizes ramp up (per/8, per/4, per/2) at the start and down again at the
// end; every chunk but the last is a multiple of `align` units.
inline std::vector<int64_t> plan_chunks(int64_t units, int64_t per, int64_t align) {
  align = std::max<int64_t>(1, align);
  auto al = [&](int64_t v) { return std::max(std::min(align, per), v / align * align); };
  const int64_t ramp[3] = {al(per / 8), al(per / 4), al(per / 2)};
  const int64_t back = ramp[0] + ramp[1] + ramp[2];
  std::vector<int64_t> sizes;
  int64_t left = units;
  auto take = [&](int64_t n) {
    n = std::min(std::max<int64_t>(n, 1), left);
    sizes.push_back(n);
    left -= n;
  };
  for (int i = 0; i < 3 && left > 0; ++i) take(ramp[i]);
  while (left > back + per) take(per);
  if (left > back) take(std::min(per, (left - back + align - 1) / align * align));
  for (int i = 2; i >= 0 && left > 0; --i) take(i == 0 ? left : ramp[i]);
  return sizes;
}

}  // namespace tfx
