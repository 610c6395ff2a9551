// Invariants of the host-buffer session's chunk plan (csrc/chunk_plan.h):
// the chunks cover the call's units exactly, none exceeds the staging slot,
// all but the last keep the alignment, and large calls start and end with
// short chunks (the copy-in and copy-out nothing else can overlap).
#include <cstdio>
#include <cstdint>
#include <vector>

#include "chunk_plan.h"

int main() {
  long checked = 0, bad = 0;
  auto fail = [&](const char* what, int64_t u, int64_t p, int64_t a) {
    if (++bad <= 10) std::printf("FAIL %s units=%lld per=%lld align=%lld\n", what, (long long)u,
                                 (long long)p, (long long)a);
  };
  for (int64_t align : {1, 4, 64}) {
    for (int64_t per : {1, 2, 7, 8, 64, 100, 4096, 4194304}) {
      if (per >= align && per % align != 0) continue;  // slots hold whole aligned chunks
      std::vector<int64_t> us;
      for (int64_t u = 1; u <= 300; ++u) us.push_back(u);
      for (int64_t m : {1, 2, 3, 5, 17}) us.push_back(m * per + 3), us.push_back(m * per);
      for (const int64_t units : us) {
        const std::vector<int64_t> c = tfx::plan_chunks(units, per, align);
        ++checked;
        int64_t sum = 0;
        for (size_t i = 0; i < c.size(); ++i) {
          sum += c[i];
          if (c[i] < 1 || c[i] > per) fail("size out of [1, per]", units, per, align);
          if (i + 1 < c.size() && per >= align && c[i] % align != 0)
            fail("unaligned chunk before the last", units, per, align);
        }
        if (sum != units) fail("chunks do not cover the units", units, per, align);
        if (per >= 64 && units >= 4 * per) {
          const int64_t short_max = std::max(align, per / 8) + align;
          if (c.front() > short_max) fail("first chunk not short", units, per, align);
          if (c.back() > short_max) fail("last chunk not short", units, per, align);
        }
      }
    }
  }
  std::printf("chunk_plan checked=%ld bad=%ld\n", checked, bad);
  return bad == 0 ? 0 : 1;
}
