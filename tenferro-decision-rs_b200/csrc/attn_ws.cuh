// attn_ws.cuh -- warp-specialised tensor-core attention for head_dim 64
// (included by attention.cu inside its anonymous namespace; uses AttnArgs,
// routed_away, analytic_range and store_out from there).
//
// Same arithmetic class as attn_tc_kernel -- S = Q K^T and P V on tcgen05 as
// 3xTF32 (hi*hi + hi*lo + lo*hi, each operand split x = tf32(x) + rest),
// online softmax in f32 -- with the work spread over roles that run
// concurrently:
//
//   warp 0      TMA: Q once, then K and V of each 64-key block into two-slot
//               rings (a K slot is freed once S of its block has been
//               computed, a V slot after PV);
//   warp 1      MMA issuer: S(j+1) is issued before PV(j);
//   warps 2-5   split: each raw tile is rewritten in place as its tf32 part
//               plus a second tile with the rest; keys outside the CTA's
//               range are zeroed; V moves into the MN-major layout the PV
//               product reads; the keep / active masks of a partial block are
//               packed into one 32-bit word per (query row, column group);
//   warps 6-13  softmax: thread = (query row, column group of 32 keys).
//
// Tensor-pipe use. An MMA of M128 N64 K8 is short next to the pipe's latency
// from one accumulation into the same TMEM columns to the next, so a block's
// MMAs are spread over independent accumulators: S over two (k-steps 0-3 and
// 4-7, summed by the softmax threads in f32), PV over the two column groups.
//
// Accumulation. The tensor cores do not accumulate in IEEE f32 (each MMA
// keeps about 22 bits below the largest exponent of the accumulator and its
// products), so PV of each block starts a fresh TMEM partial, and the softmax
// threads add the partial of block j into an f32 sum (TMEM, through
// registers) while block j + 1 is processed. A sequence of thousands of keys then stays within the f32
// tolerance (one TMEM accumulator for the whole row drifts by ~1e-4).
//
// Softmax. Each column group g keeps its own running max m_g, sum l_g and
// output O_g, so the softmax threads never exchange values inside
// the loop; the groups are merged once at the end: m = max(m_0, m_1),
// O = sum O_g e^(m_g - m), l = sum l_g e^(m_g - m). A row's running max only
// moves when a block's max exceeds it by more than 8 (natural log units);
// until then p = e^(s - m) is at most e^8, which f32 holds as exactly as
// p <= 1.
//
// TMEM (512 columns allocated, one CTA per SM): block j uses columns
// 128 (j & 1) + [0, 64) for the first S accumulator (then P hi) and + [64,
// 128) for the second (then P lo); the PV partial of group g is at 256 + 64 g
// and its f32 sum at 384 + 64 g.
// Shared memory: Q hi, Q lo (32 KB each), K slots (hi 16 KB + lo 16 KB) x 2,
// V slots the same, mask words 2 KB, keep staging 8 KB + 256 B: 203 KB.
//
// Every wait is bounded; a role that gives up raises the CTA's abort flag,
// which ends the other roles' waits; the TMA warp then waits for the copies
// it issued and the MMA warp for the MMAs it issued before TMEM is freed.

constexpr int kWsThreads = 448;
constexpr int kWsTQ = 128;                  // queries per CTA
constexpr int kWsKB = 64;                   // keys per block
constexpr uint32_t kWsQRegion = 16384;      // 128 rows x 128 bytes
constexpr uint32_t kWsKRegion = 8192;       // 64 rows x 128 bytes
constexpr uint32_t kWsQBytes = 2 * kWsQRegion;   // one of Q hi / Q lo
constexpr uint32_t kWsTile = 2 * kWsKRegion;     // one of K hi / K lo / V hi / V lo
constexpr uint32_t kWsSlot = 2 * kWsTile;        // hi + lo
constexpr uint32_t kWsOffQlo = kWsQBytes;
constexpr uint32_t kWsOffK = 2 * kWsQBytes;
constexpr uint32_t kWsOffV = kWsOffK + 2 * kWsSlot;
constexpr uint32_t kWsOffWords = kWsOffV + 2 * kWsSlot;     // [slot][group][row] u32
constexpr uint32_t kWsOffKeep = kWsOffWords + 2 * 2 * kWsTQ * 4;  // [key][query] bytes
constexpr uint32_t kWsOffActive = kWsOffKeep + kWsKB * kWsTQ;     // [key] f32
constexpr uint32_t kWsSmem = kWsOffActive + kWsKB * 4 + 1024;     // + alignment slack
constexpr float kWsRescale = 8.0f;          // natural-log headroom before m moves
constexpr uint32_t kWsStage = 68;           // output staging row stride (floats)

struct WsShared {
  uint64_t q_full, q_split;
  uint64_t k_full[2], k_split[2], k_empty[2];
  uint64_t v_full[2], v_split[2], v_empty[2];
  uint64_t s_full[2], p_ready[2];
  uint64_t o_done, o_final, drain;
  uint32_t tmem_base;
  int abort;
  int kmin, kmax;
  unsigned long long notfull;
};

// Bounded wait; also ends when another role has given up. Returns false when
// the phase did not complete (the first role to give up counts it).
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, WsShared* sh) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(&sh->abort)) return false;
    if (clock64() - t0 > kTcWait) {
      if (atomicExch(&sh->abort, 1) == 0) atomicAdd(&g_tc_wait_timeouts, 1u);
      return false;
    }
  }
  return true;
}

// ws_wait by every lane of a warp, with one answer for the warp (the TMEM
// loads and stores that follow are warp-collective).
__device__ __forceinline__ bool ws_wait_warp(uint64_t* bar, uint32_t parity, WsShared* sh) {
  return !__any_sync(0xffffffffu, !ws_wait(bar, parity, sh));
}

// Named barriers of the role groups (0 is __syncthreads).
__device__ __forceinline__ void ws_split_sync() {  // the 128 split threads
  asm volatile("bar.sync 2, 128;" ::: "memory");
}
__device__ __forceinline__ void ws_softmax_sync() {  // the 256 softmax threads
  asm volatile("bar.sync 1, 256;" ::: "memory");
}
// bar.red.or over the 256 softmax threads: every thread gets the same answer.
__device__ __forceinline__ bool ws_softmax_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

// Rewrites `bytes` of a K-major swizzled tile (128-byte rows; row r of a
// region of `rows` rows is query / key first_row + r) in place as tf32(x) and
// writes x - tf32(x) at the same offset of `lo`. Rows outside [keep_lo,
// keep_hi) become 0 in both. The swizzle only permutes 16-byte chunks inside
// a row, so the pass is elementwise. 128 threads; thread t takes chunks t,
// t + 128, ...
__device__ __forceinline__ void ws_split(uint8_t* hi, uint8_t* lo, uint32_t bytes, uint32_t rows,
                                         int64_t first_row, int64_t keep_lo, int64_t keep_hi,
                                         uint32_t t) {
  const uint32_t lo_row = uint32_t(max(int64_t(0), min(int64_t(rows), keep_lo - first_row)));
  const uint32_t hi_row = uint32_t(max(int64_t(lo_row), min(int64_t(rows), keep_hi - first_row)));
#pragma unroll 4
  for (uint32_t c = t; c < bytes / 16; c += 128) {
    const uint32_t off = c * 16;
    const uint32_t r = (off / 128) % rows;
    float4 x = *reinterpret_cast<const float4*>(hi + off);
    if (r - lo_row >= hi_row - lo_row) x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float4 h = make_float4(tf32_round_finite(x.x), tf32_round_finite(x.y),
                                 tf32_round_finite(x.z), tf32_round_finite(x.w));
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) = make_float4(__fsub_rn(x.x, h.x), __fsub_rn(x.y, h.y),
                                                       __fsub_rn(x.z, h.z), __fsub_rn(x.w, h.w));
  }
}

// The V tile of one slot: raw values as the TMA wrote them (two regions of
// 64 key rows x 32 channels, standard 128-byte swizzle: 16-byte chunk c of
// row r at chunk c ^ (r % 8)) become tf32 hi (in place) and lo, both in the
// MN-major 32-byte-atom layout the PV product reads. Thread t owns row t % 64
// of region t / 64 and reads the whole row before writing it, so the
// permutation in place is safe. Keys outside [keep_lo, keep_hi) become 0.
__device__ __forceinline__ void ws_split_v(uint8_t* hi, uint8_t* lo, int64_t first_key,
                                           int64_t keep_lo, int64_t keep_hi, uint32_t t) {
  const uint32_t r = t & 63, region = (t >> 6) * kWsKRegion;
  const int64_t key = first_key + r;
  const bool zero = key < keep_lo || key >= keep_hi;
  float4 x[8];
#pragma unroll
  for (uint32_t c = 0; c < 8; ++c) {
    x[c] = *reinterpret_cast<const float4*>(hi + region + r * 128 + ((c ^ (r & 7)) << 4));
    if (zero) x[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
#pragma unroll
  for (uint32_t c = 0; c < 8; ++c) {
    const float4 h = make_float4(tf32_round_finite(x[c].x), tf32_round_finite(x[c].y),
                                 tf32_round_finite(x[c].z), tf32_round_finite(x[c].w));
    const uint32_t off = region + sw128b32_chunk(r, c);
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) =
        make_float4(__fsub_rn(x[c].x, h.x), __fsub_rn(x[c].y, h.y), __fsub_rn(x[c].z, h.z),
                    __fsub_rn(x[c].w, h.w));
  }
}

// Keep-mask scan over the keys [lo, hi) for the queries [q0, q0 + nq): narrows
// [lo, hi) to the keys some query keeps and returns one bit per 64-key block
// (block index kj / 64 < 64) that has a (query, key) the mask drops. Every
// thread of the CTA gets the results. Eight threads read one key's 128 query
// bytes as 16-byte words (keep[q + L*(k + L*b)]: the queries of a key are
// contiguous); each thread issues its loads for ten keys before using any of
// them, and the results are reduced per warp, then once per warp in shared
// memory.
__device__ unsigned long long ws_keep_scan(const AttnArgs& a, uint32_t b, uint32_t q0,
                                           uint32_t nq, int64_t* lo, int64_t* hi,
                                           WsShared& sh) {
  if (threadIdx.x == 0) {
    sh.kmin = 0x7fffffff;
    sh.kmax = -1;
    sh.notfull = 0;
  }
  __syncthreads();
  const uint64_t L = a.length;
  const uint32_t c = threadIdx.x & 7;  // 16-query chunk of the row
  const uint32_t i0 = c * 16, i1 = min(nq, i0 + 16);
  const bool vec = L % 16 == 0 && (reinterpret_cast<uintptr_t>(a.keep) & 15) == 0 && i1 - i0 == 16;
  const uint32_t per = blockDim.x >> 3;  // keys per pass
  constexpr int U = 10;
  int kmin = 0x7fffffff, kmax = -1;
  unsigned long long nf = 0;
  if (i0 < i1) {
    for (int64_t base = *lo + (threadIdx.x >> 3); base < *hi; base += int64_t(per) * U) {
      uint4 w[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t kj = base + int64_t(u) * per;
        w[u] = make_uint4(0, 0, 0, 0);
        if (vec && kj < *hi)
          w[u] = __ldg(reinterpret_cast<const uint4*>(a.keep + uint64_t(q0) + i0 +
                                                      L * (uint64_t(kj) + L * b)));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t kj = base + int64_t(u) * per;
        if (kj >= *hi) break;
        bool any = false, all = true;
        if (vec) {
          any = (w[u].x | w[u].y | w[u].z | w[u].w) != 0;
          auto zero_byte = [](uint32_t v) { return ((v - 0x01010101u) & ~v & 0x80808080u) != 0; };
          all = !(zero_byte(w[u].x) || zero_byte(w[u].y) || zero_byte(w[u].z) || zero_byte(w[u].w));
        } else {
          const uint8_t* row = a.keep + uint64_t(q0) + L * (uint64_t(kj) + L * b);
          for (uint32_t i = i0; i < i1; ++i) {
            const bool k = row[i] != 0;
            any |= k;
            all &= k;
          }
        }
        if (any) {
          kmin = min(kmin, int(kj));
          kmax = max(kmax, int(kj));
        }
        if (!all && (kj >> 6) < 64) nf |= 1ull << (kj >> 6);
      }
    }
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  const uint32_t nf_lo = __reduce_or_sync(0xffffffffu, uint32_t(nf));
  const uint32_t nf_hi = __reduce_or_sync(0xffffffffu, uint32_t(nf >> 32));
  if ((threadIdx.x & 31) == 0) {
    if (kmax >= 0) {
      atomicMin(&sh.kmin, kmin);
      atomicMax(&sh.kmax, kmax);
    }
    const unsigned long long m = (uint64_t(nf_hi) << 32) | nf_lo;
    if (m) atomicOr(&sh.notfull, m);
  }
  __syncthreads();
  const int first = sh.kmin, last = sh.kmax;
  const unsigned long long notfull = sh.notfull;
  if (first > last) {
    *hi = *lo;
  } else {
    *lo = first;
    *hi = int64_t(last) + 1;
  }
  return ~notfull;
}

// Mask words of the 64-key block at kb for the split threads (t = query row
// of the CTA): bit c of words[g * 128 + t] is set when key kb + 32 g + c is in
// [lo, hi), the keep tensor keeps (query, key) and the key is active. The keep
// tile is first staged in shared memory with 16-byte loads (all issued before
// any is used), so that each row's 64 bits come from shared memory.
template <bool KEEP, bool ACTIVE>
__device__ __forceinline__ void ws_build_words(const AttnArgs& a, uint32_t b, uint32_t q0,
                                               uint32_t nq, int64_t kb, int64_t lo, int64_t hi,
                                               uint8_t* keep_s, float* act_s, uint32_t* words,
                                               uint32_t t) {
  const uint64_t L = a.length;
  if constexpr (KEEP) {
    const bool vec = L % 16 == 0 && (reinterpret_cast<uintptr_t>(a.keep) & 15) == 0 && nq == kWsTQ;
    uint4 w[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t idx = t + 128 * r, key = idx >> 3, c = (idx & 7) * 16;
      const int64_t kj = kb + key;
      w[r] = make_uint4(0, 0, 0, 0);
      if (kj >= lo && kj < hi) {
        const uint8_t* src = a.keep + uint64_t(q0) + c + L * (uint64_t(kj) + L * b);
        if (vec) {
          w[r] = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          uint8_t tmp[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) tmp[i] = c + i < nq ? src[i] : 0;
          memcpy(&w[r], tmp, 16);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t idx = t + 128 * r;
      *reinterpret_cast<uint4*>(keep_s + (idx >> 3) * kWsTQ + (idx & 7) * 16) = w[r];
    }
  }
  if constexpr (ACTIVE) {
    if (t < kWsKB) {
      const int64_t kj = kb + t;
      act_s[t] = kj >= lo && kj < hi ? a.active[uint64_t(b) * L + uint64_t(kj)] : 0.0f;
    }
  }
  ws_split_sync();
#pragma unroll
  for (uint32_t g = 0; g < 2; ++g) {
    uint32_t w = 0;
#pragma unroll
    for (uint32_t c = 0; c < 32; ++c) {
      const uint32_t key = 32 * g + c;
      const int64_t kj = kb + key;
      bool kept = t < nq && kj >= lo && kj < hi;
      if constexpr (KEEP) kept = kept && keep_s[key * kWsTQ + t] != 0;
      if constexpr (ACTIVE) kept = kept && act_s[key] != 0.0f;
      w |= uint32_t(kept) << c;
    }
    words[g * kWsTQ + t] = w;
  }
  ws_split_sync();  // the staging is rewritten by the next call
}

// bar.red.or over the 128 split threads (named barrier 2).
__device__ __forceinline__ bool ws_split_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v))
      : "memory");
  return r != 0;
}

// qmap: q rows with a {32, 128} box; kmap / vmap: k / v rows with a {32, 64}
// box; all three 128-byte swizzled (attention.cu encodes them).
template <bool KEEP, bool BIAS, bool ACTIVE>
__global__ void __launch_bounds__(kWsThreads, 1) attn_ws_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t ws_smem[];
  __shared__ WsShared sh;
  pdl_enter();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t q0 = blockIdx.x * kWsTQ, head = blockIdx.y, b = blockIdx.z;
  const uint32_t bh = b * a.heads + head;
  if (routed_away(a, bh)) return;
  const uint32_t L = a.length;
  const uint32_t nq = min(uint32_t(kWsTQ), L - q0);
  const uint64_t row0 = uint64_t(bh) * L;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws_smem) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* qhi = base;
  uint8_t* qlo = base + kWsOffQlo;
  uint32_t* words = reinterpret_cast<uint32_t*>(base + kWsOffWords);  // [slot][group][row]

  int64_t lo, hi;
  analytic_range(a, q0, q0 + nq - 1, &lo, &hi);
  unsigned long long full_bits = ~0ull;
  if (KEEP && lo < hi) full_bits = ws_keep_scan(a, b, q0, nq, &lo, &hi, sh);
  const int64_t kb_first = lo / kWsKB * kWsKB;
  const uint32_t nblk = kb_first < hi ? uint32_t((hi - kb_first + kWsKB - 1) / kWsKB) : 0;
  // mask words are built (and read) for block j when this holds
  auto need_words = [&](uint32_t j) {
    if (ACTIVE) return true;
    if (!KEEP) return false;
    const int64_t blk = (kb_first >> 6) + j;
    return !(blk < 64 && ((full_bits >> blk) & 1));
  };

  if (tid == 0) {
    mbar_init(&sh.q_full, 1);
    mbar_init(&sh.q_split, 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.k_split[s], 128);
      mbar_init(&sh.k_empty[s], 1);
      mbar_init(&sh.v_full[s], 1);
      mbar_init(&sh.v_split[s], 128);
      mbar_init(&sh.v_empty[s], 1);
      mbar_init(&sh.s_full[s], 1);
      mbar_init(&sh.p_ready[s], 256);
    }
    mbar_init(&sh.o_done, 1);
    mbar_init(&sh.o_final, 1);
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) tmem_alloc(&sh.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = sh.tmem_base;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0 && nblk > 0) {
      mbar_arrive_expect_tx(&sh.q_full, kWsQBytes);
      tma_load_2d(qhi, &qmap, &sh.q_full, 0, int(row0 + q0));
      tma_load_2d(qhi + kWsQRegion, &qmap, &sh.q_full, 32, int(row0 + q0));
      uint32_t kiss[2] = {0, 0}, viss[2] = {0, 0};
      for (uint32_t j = 0; j < nblk; ++j) {
        const uint32_t s = j & 1, use = j >> 1;
        const int row = int(row0 + kb_first + int64_t(j) * kWsKB);
        uint8_t* ks = base + kWsOffK + s * kWsSlot;
        uint8_t* vs = base + kWsOffV + s * kWsSlot;
        if (use > 0 && !ws_wait(&sh.k_empty[s], (use - 1) & 1, &sh)) break;
        mbar_arrive_expect_tx(&sh.k_full[s], kWsTile);
        tma_load_2d(ks, &kmap, &sh.k_full[s], 0, row);
        tma_load_2d(ks + kWsKRegion, &kmap, &sh.k_full[s], 32, row);
        ++kiss[s];
        if (use > 0 && !ws_wait(&sh.v_empty[s], (use - 1) & 1, &sh)) break;
        mbar_arrive_expect_tx(&sh.v_full[s], kWsTile);
        tma_load_2d(vs, &vmap, &sh.v_full[s], 0, row);
        tma_load_2d(vs + kWsKRegion, &vmap, &sh.v_full[s], 32, row);
        ++viss[s];
      }
      // the copies this thread issued land before the CTA can exit
      mbar_wait_bounded(&sh.q_full, 0, kTcWait);
      for (int s = 0; s < 2; ++s) {
        if (kiss[s] > 0) mbar_wait_bounded(&sh.k_full[s], (kiss[s] - 1) & 1, kTcWait);
        if (viss[s] > 0) mbar_wait_bounded(&sh.v_full[s], (viss[s] - 1) & 1, kTcWait);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t id_s = idesc_tf32(kWsTQ, kWsKB);
      constexpr uint32_t id_o = idesc_tf32_bmn(kWsTQ, 64);
      // S(j): chain A (k-steps 0-3) and chain B (4-7) issued alternately
      auto issue_s = [&](uint32_t j) -> bool {
        const uint32_t s = j & 1;
        if (!ws_wait(&sh.k_split[s], (j >> 1) & 1, &sh)) return false;
        tc_fence_after();
        const uint32_t dst = tm + 128 * s;
        // descriptors built once; an offset moves the start address field
        // (address >> 4, no carry out of its 14 bits inside shared memory)
        const uint64_t dqh = smem_desc_sw128(smem_addr(qhi));
        const uint64_t dql = smem_desc_sw128(smem_addr(qlo));
        const uint64_t dkh = smem_desc_sw128(smem_addr(base + kWsOffK + s * kWsSlot));
        const uint64_t dkl = dkh + (kWsTile >> 4);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (uint32_t prod = 0; prod < 3; ++prod) {
#pragma unroll
            for (uint32_t ch = 0; ch < 2; ++ch) {
              const uint64_t a_q = (prod == 2 ? dql : dqh) + ((ch * kWsQRegion + kk * 32) >> 4);
              const uint64_t b_k = (prod == 1 ? dkl : dkh) + ((ch * kWsKRegion + kk * 32) >> 4);
              mma_tf32_ss(dst + 64 * ch, a_q, b_k, id_s, (kk > 0 || prod > 0) ? 1u : 0u);
            }
          }
        }
        mma_commit(&sh.s_full[s]);
        mma_commit(&sh.k_empty[s]);  // K slot free once these MMAs have read it
        return true;
      };
      bool ok = ws_wait(&sh.q_split, 0, &sh) && issue_s(0);
      for (uint32_t j = 0; ok && j < nblk; ++j) {
        if (j + 1 < nblk && !issue_s(j + 1)) break;
        const uint32_t s = j & 1;
        if (!ws_wait(&sh.p_ready[s], (j >> 1) & 1, &sh) ||
            !ws_wait(&sh.v_split[s], (j >> 1) & 1, &sh))
          break;
        tc_fence_after();
        // PV(j): a fresh partial per column group, the two groups alternating
        const uint32_t ph = tm + 128 * s, pl = ph + 64;
        const uint64_t dvh = smem_desc_sw128b32_mn(smem_addr(base + kWsOffV + s * kWsSlot),
                                                   kWsKRegion);
        const uint64_t dvl = dvh + (kWsTile >> 4);
#pragma unroll
        for (uint32_t kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (uint32_t prod = 0; prod < 3; ++prod) {
#pragma unroll
            for (uint32_t g = 0; g < 2; ++g) {
              const uint32_t ks = 4 * g + kk;
              const uint32_t a_t = (prod == 2 ? pl : ph) + ks * 8;
              const uint64_t b_v = (prod == 1 ? dvl : dvh) + ((ks * 1024) >> 4);
              mma_tf32_ts(tm + 256 + 64 * g, a_t, b_v, id_o, (kk > 0 || prod > 0) ? 1u : 0u);
            }
          }
        }
        mma_commit(&sh.o_done);
        mma_commit(&sh.v_empty[s]);
        if (j + 1 == nblk) mma_commit(&sh.o_final);
      }
      // every MMA issued has completed before TMEM is freed
      mma_commit(&sh.drain);
      mbar_wait_bounded(&sh.drain, 0, kTcWait);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ---- split: tf32 hi in place, lo beside it; mask words of partial blocks ----
    const uint32_t t = tid - 64;  // 0..127, also the query row of the mask words
    if (nblk > 0) {
      // every decision to go on is taken by all 128 split threads together
      // (they meet at named barriers)
      bool ok = !ws_split_any(!ws_wait(&sh.q_full, 0, &sh));
      if (ok) {  // rows past the sequence (another head's queries) become 0
        ws_split(qhi, qlo, kWsQBytes, kWsTQ, q0, q0, int64_t(q0) + nq, t);
        fence_proxy_async_smem();
        mbar_arrive(&sh.q_split);
      }
      for (uint32_t j = 0; ok && j < nblk; ++j) {
        const uint32_t s = j & 1, ph = (j >> 1) & 1;
        const int64_t kb = kb_first + int64_t(j) * kWsKB;
        uint8_t* ks = base + kWsOffK + s * kWsSlot;
        uint8_t* vs = base + kWsOffV + s * kWsSlot;
        if (ws_split_any(!ws_wait(&sh.k_full[s], ph, &sh))) break;
        ws_split(ks, ks + kWsTile, kWsTile, kWsKB, kb, lo, hi, t);
        // k_split(j) follows the softmax of block j - 2: it has finished with
        // this word slot, and no softmax thread still waits for k_split of
        // block j - 2 (so k_split never runs two phases ahead of a waiter)
        if (j >= 2 && ws_split_any(!ws_wait(&sh.p_ready[s], ((j - 2) >> 1) & 1, &sh))) break;
        if (need_words(j))
          ws_build_words<KEEP, ACTIVE>(a, b, q0, nq, kb, lo, hi, base + kWsOffKeep,
                                       reinterpret_cast<float*>(base + kWsOffActive),
                                       words + s * 2 * kWsTQ, t);
        fence_proxy_async_smem();
        mbar_arrive(&sh.k_split[s]);
        if (ws_split_any(!ws_wait(&sh.v_full[s], ph, &sh))) break;
        ws_split_v(vs, vs + kWsTile, kb, lo, hi, t);
        fence_proxy_async_smem();
        mbar_arrive(&sh.v_split[s]);
      }
    }
  } else {
    // ---- softmax: thread = (query row, column group g of 32 keys) ----
    const uint32_t g = (warp - 6) >> 2, quarter = warp & 3;
    const uint32_t row = quarter * 32 + lane;
    const uint32_t lane_off = (quarter * 32) << 16;
    const uint32_t tO = tm + 256 + 64 * g + lane_off;    // this group's PV partial
    const uint32_t tAcc = tm + 384 + 64 * g + lane_off;  // its f32 sum of the partials
    const int64_t qi = int64_t(q0) + row;
    // this row's keys by the analytic conditions and the CTA's range
    int64_t r_lo = lo, r_hi = qi < L ? hi : lo;
    if (a.causal) r_hi = min(r_hi, qi + 1);
    if (a.window >= 0) {
      r_lo = max(r_lo, qi - a.window);
      r_hi = min(r_hi, qi + a.window + 1);
    }
    if (a.valid_len >= 0) r_hi = min(r_hi, a.valid_len);
    if (r_hi < r_lo) r_hi = r_lo;
    constexpr float kLog2e = 1.44269504088896341f;
    float m = -INFINITY, l = 0.0f;  // running max (natural units), sum
    bool inf_row = false, failed = false;
    for (uint32_t j = 0; j < nblk; ++j) {
      const uint32_t s = j & 1, ph = (j >> 1) & 1;
      const int64_t k0 = kb_first + int64_t(j) * kWsKB + 32 * g;  // key of column 0
      const bool nw = need_words(j);
      if (!ws_wait_warp(&sh.s_full[s], ph, &sh) ||
          (nw && !ws_wait_warp(&sh.k_split[s], ph, &sh))) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t word = nw ? words[(s * 2 + g) * kWsTQ + row] : ~0u;
      const int64_t c_lo64 = max(int64_t(0), min(int64_t(32), r_lo - k0));
      const int64_t c_hi64 = max(c_lo64, min(int64_t(32), r_hi - k0));
      const uint32_t c_lo = uint32_t(c_lo64), c_span = uint32_t(c_hi64 - c_lo64);
      const uint32_t tA = tm + 128 * s + 32 * g + lane_off, tB = tA + 64;
      float sv[32];
      {
        float sa[32], sb[32];
        tmem_ld16(tA, sa);
        tmem_ld16(tA + 16, sa + 16);
        tmem_ld16(tB, sb);
        tmem_ld16(tB + 16, sb + 16);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __fmul_rn(__fadd_rn(sa[i], sb[i]), a.scale);
      }
      float mb = -INFINITY;
      if (!BIAS && c_span == 32 && word == ~0u) {  // every key of the span kept
#pragma unroll
        for (uint32_t c = 0; c < 32; ++c) mb = fmaxf(mb, sv[c]);
      } else {
#pragma unroll
        for (uint32_t c = 0; c < 32; ++c) {
          float sc = sv[c];
          const bool kept = c - c_lo < c_span && ((word >> c) & 1);
          if constexpr (BIAS)  // read only for kept keys: those lie inside the tensor
            if (kept) sc = __fadd_rn(sc, a.bias[uint64_t(qi) + uint64_t(L) * (uint64_t(k0 + c) + uint64_t(L) * b)]);
          sc = kept ? sc : -INFINITY;
          if constexpr (BIAS) sc = sc == sc ? sc : -INFINITY;  // a NaN bias: nothing
          sv[c] = sc;
          mb = fmaxf(mb, sc);
        }
      }
      // q, k, v are finite here (checked before launch): a score is finite
      // unless q.k * scale (+ bias) overflows; a row with a +inf score takes
      // the empty value at the end (its values meanwhile do not matter: the
      // rows of the products are independent)
      inf_row |= mb == INFINITY;
      // move the running max only when the block's max is well above it
      float mn = m, corr = 1.0f;
      if (mb > m) {
        if (m == -INFINITY) {
          mn = mb;  // nothing of this row has been summed yet
        } else if (mb > m + kWsRescale) {
          mn = mb;
          corr = expf(m - mb);
        }
      }
      // p = e^(s - mn) = 2^(s log2e - mn log2e): one FMA and the hardware 2^x
      // (relative error ~2^-22), split into tf32 hi (over the first S
      // accumulator) and lo (over the second)
      const float mnl = mn == -INFINITY ? 0.0f : __fmul_rn(mn, kLog2e);
      float ps = 0.0f;
#pragma unroll
      for (uint32_t h = 0; h < 32; h += 16) {
        float phi[16], plo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float p;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p) : "f"(__fmaf_rn(sv[h + i], kLog2e, -mnl)));
          ps = __fadd_rn(ps, p);
          phi[i] = tf32_round_finite(p);
          plo[i] = __fsub_rn(p, phi[i]);
        }
        tmem_st16(tA + h, phi);
        tmem_st16(tB + h, plo);
      }
      l = __fmaf_rn(l, corr, ps);
      m = mn;
      // the partial of block j - 1 goes into the f32 sum before PV(j)
      // overwrites it: acc = (acc + partial) * corr. The parity wait is
      // exact: PV(j-2) has completed (S(j), whose completion this thread has
      // seen, was issued after it) and PV(j) cannot start before this
      // thread's P(j).
      if (j > 0) {
        if (!ws_wait_warp(&sh.o_done, (j - 1) & 1, &sh)) {
          failed = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (uint32_t c = 0; c < 64; c += 32) {
          float pv[32], av[32];
          tmem_ld16(tO + c, pv);
          tmem_ld16(tO + c + 16, pv + 16);
          if (j > 1) {
            tmem_ld16(tAcc + c, av);
            tmem_ld16(tAcc + c + 16, av + 16);
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            av[i] = __fmul_rn(j > 1 ? __fadd_rn(av[i], pv[i]) : pv[i], corr);
          tmem_st16(tAcc + c, av);
          tmem_st16(tAcc + c + 16, av + 16);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sh.p_ready[s]);
    }
    // o_final, not o_done: PV(nblk - 2) is issued after S(nblk - 1), so a
    // parity wait on o_done could see the phase of PV(nblk - 2) still open
    // and take it for the completed phase before
    if (!failed && nblk > 0) {
      failed = !ws_wait_warp(&sh.o_final, 0, &sh);
      tc_fence_after();
    }
    if (!ws_softmax_any(failed)) {
      // merge the two column groups through the (now idle) K ring: group g
      // keeps its own half of the channels (acc + last partial) and hands
      // the other half over
      float* xo = reinterpret_cast<float*>(base + kWsOffK);  // [group][row][33]
      float* xm = xo + 2 * kWsTQ * 33;
      float* xl = xm + 2 * kWsTQ;
      int* xi = reinterpret_cast<int*>(xl + 2 * kWsTQ);
      const uint32_t other = 1 - g;
      float own[32];
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) {
        float v[32];
        if (nblk > 0) {  // uniform over the CTA: every lane joins the .aligned loads
          float av[32];
          tmem_ld16(tO + 32 * h, v);
          tmem_ld16(tO + 32 * h + 16, v + 16);
          if (nblk > 1) {
            tmem_ld16(tAcc + 32 * h, av);
            tmem_ld16(tAcc + 32 * h + 16, av + 16);
          }
          tmem_wait_ld();
          if (nblk > 1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __fadd_rn(av[i], v[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.0f;
        }
        if (h == g) {
#pragma unroll
          for (int i = 0; i < 32; ++i) own[i] = v[i];
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) xo[(g * kWsTQ + row) * 33 + i] = v[i];
        }
      }
      xm[g * kWsTQ + row] = m;
      xl[g * kWsTQ + row] = l;
      xi[g * kWsTQ + row] = inf_row;
      ws_softmax_sync();
      const float mo = xm[other * kWsTQ + row], lo_o = xl[other * kWsTQ + row];
      const bool inf_any = inf_row || xi[other * kWsTQ + row] != 0;
      const float mx = fmaxf(m, mo);
      const float fs = m == -INFINITY ? 0.0f : expf(m - mx);
      const float fo = mo == -INFINITY ? 0.0f : expf(mo - mx);
      const float lsum = __fadd_rn(__fmul_rn(l, fs), __fmul_rn(lo_o, fo));
      const bool empty = nblk == 0 || lsum == 0.0f || inf_any;
      const float ev = a.empty_nan ? NAN : 0.0f;
      const float rl = __frcp_rn(lsum);
#pragma unroll
      for (uint32_t c = 0; c < 32; ++c) {
        const float v = __fadd_rn(__fmul_rn(own[c], fs),
                                  __fmul_rn(xo[(other * kWsTQ + row) * 33 + c], fo));
        own[c] = empty ? ev : __fmul_rn(v, rl);
      }
      // feature-contiguous output rows (the Laya block's and the attention
      // core's layouts): staged in the idle V ring, then written as whole
      // 256-byte rows; any other layout element by element
      const bool vec = a.out_feat == 1 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                       a.out_tok % 4 == 0 && a.out_batch % 4 == 0 &&
                       (!a.gate || ((reinterpret_cast<uintptr_t>(a.gate) & 15) == 0 &&
                                    a.gate_offset % 4 == 0));
      if (vec) {
        float* stage = reinterpret_cast<float*>(base + kWsOffV);  // [row][kWsStage]
#pragma unroll
        for (uint32_t c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(stage + row * kWsStage + 32 * g + c) =
              make_float4(own[c], own[c + 1], own[c + 2], own[c + 3]);
        ws_softmax_sync();
        const uint32_t ts = tid - 192;  // 0..255
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
          const uint32_t idx = ts + 256 * i, r = idx >> 4, c4 = (idx & 15) * 4;
          const uint32_t qr = q0 + r;
          if (qr >= L) continue;
          float4 v4 = *reinterpret_cast<const float4*>(stage + r * kWsStage + c4);
          const int64_t oi = int64_t(qr) * a.out_tok + int64_t(head) * 64 + c4 +
                             int64_t(b) * a.out_batch;
          if (a.gate) {
            const float4 g4 = *reinterpret_cast<const float4*>(a.gate + a.gate_offset + oi);
            auto sg = [](float x, float gv) {
              return __fmul_rn(x, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv))));
            };
            v4 = make_float4(sg(v4.x, g4.x), sg(v4.y, g4.y), sg(v4.z, g4.z), sg(v4.w, g4.w));
          }
          *reinterpret_cast<float4*>(a.out + oi) = v4;
        }
      } else if (qi < L) {
#pragma unroll
        for (uint32_t c = 0; c < 32; ++c)
          store_out(a, b, uint32_t(qi), uint64_t(head) * 64 + 32 * g + c, own[c]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_free(tm, 512);
}
