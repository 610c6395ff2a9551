// Exhaustive host check: the product's branch-free erf_mlx / gelu_mlx
// (tenferro-decision-rs_b200/csrc/tfx_math.h, compiled here by the host
// compiler with -ffp-contract=off) against the oracle's literal restatement
// of crates/cpu-kernels/src/lib.rs:449-511, bit for bit, over every f32 bit
// pattern in [begin, end) with the given stride. Prints one summary line and
// exits non-zero on any mismatch.
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "oracle.h"
#include "tfx_math.h"

static bool same(float a, float b) {
  if (a != a && b != b) return true;
  uint32_t x, y;
  memcpy(&x, &a, 4);
  memcpy(&y, &b, 4);
  return x == y;
}

int main(int argc, char** argv) {
  const uint64_t stride = argc > 1 ? strtoull(argv[1], nullptr, 10) : 1;
  const uint64_t begin = 0, end = uint64_t(1) << 32;
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  std::atomic<uint64_t> bad_erf{0}, bad_gelu{0}, checked{0};
  std::atomic<uint64_t> first_bad{~uint64_t(0)};
  std::vector<std::thread> pool;
  const uint64_t chunk = (end - begin) / nt + 1;
  for (unsigned t = 0; t < nt; ++t) {
    pool.emplace_back([&, t] {
      uint64_t lo = begin + t * chunk, hi = lo + chunk < end ? lo + chunk : end;
      lo += (stride - (lo - begin) % stride) % stride;
      uint64_t be = 0, bg = 0, n = 0;
      for (uint64_t b = lo; b < hi; b += stride) {
        uint32_t bits = uint32_t(b);
        float x;
        memcpy(&x, &bits, 4);
        ++n;
        if (!same(tfx::math::erf_mlx(x), orc_erf_f32(x))) {
          ++be;
          uint64_t cur = first_bad.load();
          while (b < cur && !first_bad.compare_exchange_weak(cur, b)) {}
        }
        if (!same(tfx::math::gelu_mlx(x), orc_gelu_erf_f32(x))) ++bg;
      }
      bad_erf += be;
      bad_gelu += bg;
      checked += n;
    });
  }
  for (auto& th : pool) th.join();
  printf("checked=%llu erf_mismatch=%llu gelu_mismatch=%llu first_bad_bits=0x%llx\n",
         (unsigned long long)checked.load(), (unsigned long long)bad_erf.load(),
         (unsigned long long)bad_gelu.load(), (unsigned long long)first_bad.load());
  return (bad_erf.load() == 0 && bad_gelu.load() == 0) ? 0 : 1;
}
