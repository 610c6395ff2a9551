// attn_ws.cuh -- tensor-core attention for head_dim 64 over pre-split
// operand tiles (included by attention.cu inside its anonymous namespace;
// uses AttnArgs, routed_away, analytic_range and store_out from there).
//
// S = Q K^T and P V run on tcgen05 as 3xTF32 (hi*hi + hi*lo + lo*hi, each
// operand split x = tf32(x) + rest; the dropped lo*lo term is ~2^-22
// relative), the online softmax in f32. The design follows two measured
// facts of the tensor cores:
//   * one thread issues at most about one tcgen05.mma every ~100 cycles,
//     whatever N is; M128 N64 K8 products (the only N that P V of head_dim 64
//     has) are therefore issue-bound, and several issuing threads multiply
//     the rate (two measured at 1.8x);
//   * the f32 accumulation of an MMA keeps about 22 bits below the largest
//     exponent involved, so a long sum in one TMEM accumulator drifts.
//
// Operands. attn_img_split_kernel writes q, k and v once as tf32 hi / lo
// "tile images": byte for byte the shared-memory layout the MMAs read, so the
// attention kernel moves each tile with one bulk copy and does no conversion:
//   Q: 128-query tiles, K-major 128-byte swizzle (16-byte chunk c of row r at
//      c ^ (r % 8)), two 32-channel regions of 16 KB, hi then lo (64 KB);
//   K: 64-key tiles, the same layout, regions of 8 KB, hi then lo (32 KB);
//   V: 64-key tiles, rows = keys, MN-major in the 32-byte-atom swizzle that
//      MN-major tf32 operands need (32-byte granule g of row r at g ^ (r % 4)),
//      regions of 8 KB, hi then lo (32 KB).
// Rows past the sequence are zero, so no tile holds another head's values.
//
// Masks. The keep and active masks do not depend on the head, so
// attn_keep_digest_kernel condenses them once per call: per (batch, query
// tile, 64-key block) one 32-bit word per (query row, column group) and a
// summary byte (some / every (query, key) kept). A CTA narrows its key range
// from the summary row and its softmax threads load their words directly.
//
// Roles (12 warps):
//   warp 0      bulk copies of V (a two-slot ring) and P V of column group 1
//               for every block;
//   warps 1-3   MMA issuers: issuer p computes S(j) and P V of column group
//               0 of the blocks j = p mod 3 (both halves of P V run at once:
//               one thread issues at most one MMA per ~100 cycles); S(j + 3)
//               waits until both halves of P V(j) have read buffer p; each
//               issuer loads its own K tiles (Q once, by thread 0) into its
//               own K slot as soon as its S has read the slot;
//   warps 4-11  softmax: thread = (query row, column group g of 32 keys).
//
// TMEM (512 columns, one CTA per SM): block j (p = j % 3) has S, then P hi,
// in columns 128 p + [0, 64), P lo in 128 p + [64, 128); the P V partial of
// group g is at 384 + 64 g, fresh for every block. The softmax threads add
// the partial of block j into f32 registers while block j + 1 is processed
// (before P V(j + 1), which waits for them, overwrites it), so a sequence of
// any length stays within the f32 tolerance.
//
// Softmax. Each column group g keeps its own running max m_g, sum l_g and
// output O_g, so the softmax threads never exchange values inside the loop;
// the groups are merged once at the end: m = max(m_0, m_1),
// O = sum O_g e^(m_g - m), l = sum l_g e^(m_g - m). A row's running max only
// moves when a block's max exceeds it by more than 8 (natural log units);
// until then p = e^(s - m) is at most e^8, which f32 holds as exactly as
// p <= 1, and nothing is rescaled.
//
// Every wait is bounded; a role that gives up raises the CTA's abort flag,
// which ends the other roles' waits; the copy warp then waits for the copies
// it issued and each issuer for its MMAs before TMEM is freed.

constexpr int kWsThreads = 384;
constexpr uint32_t kWsIssuers = 3;          // MMA issuers (block j -> issuer j % 3)
constexpr uint32_t kWsOffQlo = kWsQPlane;
constexpr uint32_t kWsOffK = 2 * kWsQPlane;
constexpr uint32_t kWsOffV = kWsOffK + 3 * kWsSlot;  // K: one slot per issuer
constexpr uint32_t kWsSmem = kWsOffV + 2 * kWsSlot + 1024;  // + alignment slack
constexpr float kWsRescale = 8.0f;          // natural-log headroom before m moves
constexpr uint32_t kWsStage = 68;           // output staging row stride (floats)

struct WsShared {
  uint64_t q_full;
  uint64_t v_empty[2];  // per V slot (block j -> slot j % 2)
  // per issuer (block j -> issuer and K slot j % 3)
  uint64_t k_full[kWsIssuers], k_empty[kWsIssuers], v_full[kWsIssuers], s_full[kWsIssuers];
  uint64_t p_ready[kWsIssuers], o_done[kWsIssuers], drain[kWsIssuers + 1];
  uint32_t tmem_base;
  int abort;
  int kmin, kmax;
};

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global memory into shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

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

// The 256 softmax threads: named barrier 1, and bar.red.or (every thread
// gets the same answer).
__device__ __forceinline__ void ws_softmax_sync() {
  asm volatile("bar.sync 1, 256;" ::: "memory");
}
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

// One thread per (head, row of the padded query length lq, 4 channels): q, k
// and v of that row (0 past the sequence; k and v only for rows below lk)
// split into tf32 hi / lo and written into the tile images. flags[bh] = 1
// (when flags is given) if a value of the head is non-finite or beyond the
// largest tf32: the f32 kernel takes that head.
__global__ void __launch_bounds__(256) attn_img_split_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    uint8_t* __restrict__ qimg, uint8_t* __restrict__ kimg, uint8_t* __restrict__ vimg,
    uint32_t L, uint32_t lq, uint32_t lk, uint64_t total, uint8_t* flags) {
  pdl_enter();
  const uint32_t nqt = lq / kWsTQ, nkt = lk / kWsKB;
  for (uint64_t n = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; n < total;
       n += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t ch = uint32_t(n & 15) * 4;
    const uint64_t rest = n >> 4;
    const uint64_t bh = rest / lq;
    const uint32_t r = uint32_t(rest - bh * lq);
    const uint64_t src = (bh * L + r) * 64 + ch;
    bool bad = false;
    auto put = [&](const float* x_src, uint8_t* img, uint64_t tile_bytes, uint32_t off) {
      float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (r < L) x = ld_stream(reinterpret_cast<const float4*>(x_src + src));
      float4 h, lo;
      img_split4(x, &h, &lo, &bad);
      *reinterpret_cast<float4*>(img + off) = h;
      *reinterpret_cast<float4*>(img + tile_bytes / 2 + off) = lo;
    };
    put(q, qimg + (bh * nqt + r / kWsTQ) * (2 * kWsQPlane), 2 * kWsQPlane,
        img_kmajor_off(r % kWsTQ, ch, kWsQRegion));
    if (r < lk) {
      const uint64_t kt = (bh * nkt + r / kWsKB) * kWsSlot;
      put(k, kimg + kt, kWsSlot, img_kmajor_off(r % kWsKB, ch, kWsKRegion));
      put(v, vimg + kt, kWsSlot, img_v_off(r % kWsKB, ch));
    }
    if (bad && flags) flags[bh] = 1;
  }
}

// Zeroes the rows past the sequence (L .. lq - 1 of Q, L .. lk - 1 of K and
// V; hi and lo) in the last tile of every head's images, for images that a
// kernel writing only the rows below L (the Laya prep kernel) produced.
__global__ void __launch_bounds__(256) attn_img_pad_kernel(uint8_t* __restrict__ qimg,
                                                           uint8_t* __restrict__ kimg,
                                                           uint8_t* __restrict__ vimg, uint32_t L,
                                                           uint32_t lq, uint32_t lk,
                                                           uint64_t total) {
  pdl_enter();
  const uint32_t pad = lq - L, nqt = lq / kWsTQ, nkt = lk / kWsKB;
  const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (uint64_t n = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; n < total;
       n += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t ch = uint32_t(n & 15) * 4;
    const uint64_t rest = n >> 4, bh = rest / pad;
    const uint32_t r = L + uint32_t(rest - bh * pad);
    uint8_t* qt = qimg + (bh * nqt + r / kWsTQ) * (2 * kWsQPlane);
    const uint32_t oq = img_kmajor_off(r % kWsTQ, ch, kWsQRegion);
    *reinterpret_cast<float4*>(qt + oq) = z;
    *reinterpret_cast<float4*>(qt + kWsQPlane + oq) = z;
    if (r < lk) {
      const uint64_t kv = (bh * nkt + r / kWsKB) * kWsSlot;
      const uint32_t ok = img_kmajor_off(r % kWsKB, ch, kWsKRegion), ov = img_v_off(r % kWsKB, ch);
      *reinterpret_cast<float4*>(kimg + kv + ok) = z;
      *reinterpret_cast<float4*>(kimg + kv + kWsTile + ok) = z;
      *reinterpret_cast<float4*>(vimg + kv + ov) = z;
      *reinterpret_cast<float4*>(vimg + kv + kWsTile + ov) = z;
    }
  }
}

// Bit i of the result: byte i of the 16 bytes w is non-zero.
__device__ __forceinline__ uint32_t nonzero_bytes16(uint4 w) {
  auto nib = [](uint32_t x) {
    const uint32_t t = (((x & 0x7f7f7f7fu) + 0x7f7f7f7fu) | x) & 0x80808080u;  // byte MSB = non-zero
    const uint32_t b = t >> 7;                                                   // bits 0, 8, 16, 24
    return (b | (b >> 7) | (b >> 14) | (b >> 21)) & 0xFu;
  };
  return nib(w.x) | (nib(w.y) << 4) | (nib(w.z) << 8) | (nib(w.w) << 12);
}

// Transposes the 32 x 32 bit matrix whose row i is lane i's x: afterwards
// bit j of lane i is bit i of lane j's input. Five exchange stages: lanes i
// and i ^ s swap the off-diagonal s x s blocks of each 2s x 2s block.
__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x, uint32_t lane) {
  const uint32_t masks[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const uint32_t sft = 16u >> k, m = masks[k];
    const uint32_t y = __shfl_xor_sync(0xffffffffu, x, sft);
    x = (lane & sft) ? ((x & ~m) | ((y & ~m) >> sft)) : ((x & m) | ((y & m) << sft));
  }
  return x;
}

// Digest of the keep / active masks, the same for every head: one warp per
// (64-key block kt, 128-query tile qt, batch b) writes
//   words[((b * nqt + qt) * nkt + kt) * 256 + 128 g + row]: bit c set when
//     key 64 kt + 32 g + c lies in the tile's analytic range, the keep tensor
//     keeps (query 128 qt + row, key) and the key is active;
//   summary[(b * nqt + qt) * nkt + kt]: bit 0 = some (query, key) of the block
//     is kept, bit 1 = every (query, key) of the block inside the analytic
//     range is kept (the attention kernel then needs no words).
// Lane c reads the 128 query bytes of keys 64 kt + c and 64 kt + 32 + c
// (contiguous in keep[q + L*(k + L*b)]) as sixteen 16-byte loads, turns them
// into 32-row masks, and a bit transpose of each 32 x 32 block leaves row r's
// word in lane r.
__global__ void __launch_bounds__(32) attn_keep_digest_kernel(AttnArgs a, uint32_t nqt,
                                                              uint32_t nkt, uint32_t* words,
                                                              uint8_t* summary) {
  pdl_enter();
  // nothing that runs next reads the digest before its own wait: the Laya
  // block's prep kernel (which does not use it) starts at once and overlaps
  pdl_launch_dependents();
  const uint32_t kt = blockIdx.x, qt = blockIdx.y, b = blockIdx.z, lane = threadIdx.x;
  const uint64_t L = a.length;
  const uint32_t q0 = qt * kWsTQ, nq = min(uint32_t(kWsTQ), uint32_t(L) - q0);
  int64_t lo, hi;
  analytic_range(a, q0, q0 + nq - 1, &lo, &hi);
  const int64_t kb = int64_t(kt) * kWsKB;
  const bool vec = a.keep && L % 16 == 0 && (reinterpret_cast<uintptr_t>(a.keep) & 15) == 0 &&
                   nq == kWsTQ;
  bool kin[2], kon[2];
  uint4 w[2][8];
#pragma unroll
  for (uint32_t g = 0; g < 2; ++g) {
    const int64_t kj = kb + 32 * g + lane;
    kin[g] = kj >= lo && kj < hi;
    kon[g] = kin[g];
    if (a.active && kon[g]) kon[g] = a.active[uint64_t(b) * L + uint64_t(kj)] != 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) w[g][i] = make_uint4(0, 0, 0, 0);
    if (vec && kon[g]) {
      const uint4* src = reinterpret_cast<const uint4*>(a.keep + uint64_t(q0) +
                                                        L * (uint64_t(kj) + L * b));
#pragma unroll
      for (int i = 0; i < 8; ++i) w[g][i] = __ldg(src + i);
    }
  }
  uint32_t* out = words + ((uint64_t(b) * nqt + qt) * nkt + kt) * 256;
  bool any = false, all = true;
#pragma unroll
  for (uint32_t g = 0; g < 2; ++g) {
    const int64_t kj = kb + 32 * g + lane;
    const uint32_t in_keys = __ballot_sync(0xffffffffu, kin[g]);  // keys of the analytic range
#pragma unroll
    for (int rc = 0; rc < 4; ++rc) {
      const uint32_t n = nq > 32u * rc ? min(32u, nq - 32u * rc) : 0u;
      const uint32_t rows = n == 32 ? ~0u : ((1u << n) - 1u);
      uint32_t rm = 0;  // bit r: query row 32 rc + r kept for this lane's key
      if (kon[g]) {
        if (!a.keep) {
          rm = rows;
        } else if (vec) {
          rm = nonzero_bytes16(w[g][2 * rc]) | (nonzero_bytes16(w[g][2 * rc + 1]) << 16);
        } else {
          const uint8_t* src = a.keep + uint64_t(q0) + L * (uint64_t(kj) + L * b);
          for (uint32_t r = 0; r < n; ++r)
            if (src[32 * rc + r] != 0) rm |= 1u << r;
        }
      }
      const uint32_t word = warp_transpose32(rm, lane);
      out[g * kWsTQ + 32 * rc + lane] = word;
      const bool row_valid = 32u * rc + lane < nq;
      any |= word != 0;
      all &= !row_valid || (word & in_keys) == in_keys;
    }
  }
  any = __any_sync(0xffffffffu, any);
  all = __all_sync(0xffffffffu, all);
  if (lane == 0) summary[(uint64_t(b) * nqt + qt) * nkt + kt] = uint8_t(any) | uint8_t(all) << 1;
}

// qimg / kimg / vimg: the tile images of attn_img_split_kernel, nkt key tiles
// per head (gridDim.x query tiles). MASK: a keep or active mask is given, and
// words / summary are its digest (attn_keep_digest_kernel).
template <bool MASK, bool BIAS>
__global__ void __launch_bounds__(kWsThreads, 1) attn_ws_kernel(
    const uint8_t* __restrict__ qimg, const uint8_t* __restrict__ kimg,
    const uint8_t* __restrict__ vimg, uint32_t nkt, const uint32_t* __restrict__ words,
    const uint8_t* __restrict__ summary, AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t ws_smem[];
  __shared__ WsShared sh;
  pdl_enter();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t q0 = blockIdx.x * kWsTQ, head = blockIdx.y, b = blockIdx.z;
  const uint32_t bh = b * a.heads + head;
  if (routed_away(a, bh)) return;
  const uint32_t L = a.length;
  const uint32_t nq = min(uint32_t(kWsTQ), L - q0);
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws_smem) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* qhi = base;

  if (tid == 0) {
    mbar_init(&sh.q_full, 1);
    for (int s = 0; s < 2; ++s) mbar_init(&sh.v_empty[s], 2);  // both halves of P V
    for (uint32_t q = 0; q < kWsIssuers; ++q) {
      mbar_init(&sh.k_full[q], 1);
      mbar_init(&sh.k_empty[q], 1);
      mbar_init(&sh.v_full[q], 1);
      mbar_init(&sh.s_full[q], 1);
      mbar_init(&sh.p_ready[q], 256);
      mbar_init(&sh.o_done[q], 2);  // both halves of P V
    }
    for (uint32_t q = 0; q <= kWsIssuers; ++q) mbar_init(&sh.drain[q], 1);
    sh.abort = 0;
    sh.kmin = 0x7fffffff;
    sh.kmax = -1;
    mbar_init_fence();
  }
  __syncthreads();
  // Q travels while the keep mask is scanned
  if (tid == 0) {
    mbar_arrive_expect_tx(&sh.q_full, 2 * kWsQPlane);
    bulk_load(qhi, qimg + (uint64_t(bh) * gridDim.x + blockIdx.x) * (2 * kWsQPlane),
              2 * kWsQPlane, &sh.q_full);
  }

  int64_t lo, hi;
  analytic_range(a, q0, q0 + nq - 1, &lo, &hi);
  // the digest of this (batch, query tile): its key blocks' summary bytes
  // and mask words
  const uint64_t drow = uint64_t(b) * gridDim.x + blockIdx.x;
  const uint8_t* srow = MASK ? summary + drow * nkt : nullptr;
  const uint32_t* wrow = MASK ? words + drow * nkt * 256 : nullptr;
  if (MASK && lo < hi) {  // narrow [lo, hi) to the blocks that keep some (query, key)
    int first = 0x7fffffff, last = -1;
    for (int64_t kt = lo / kWsKB + tid; kt * kWsKB < hi; kt += kWsThreads)
      if (__ldg(srow + kt) & 1) {
        first = min(first, int(kt));
        last = max(last, int(kt));
      }
    first = __reduce_min_sync(0xffffffffu, first);
    last = __reduce_max_sync(0xffffffffu, last);
    if (lane == 0 && last >= 0) {
      atomicMin(&sh.kmin, first);
      atomicMax(&sh.kmax, last);
    }
    __syncthreads();
    if (sh.kmax < 0) {
      hi = lo;
    } else {
      lo = max(lo, int64_t(sh.kmin) * kWsKB);
      hi = min(hi, (int64_t(sh.kmax) + 1) * kWsKB);
    }
  }
  const int64_t kb_first = lo / kWsKB * kWsKB;
  const uint32_t nblk = kb_first < hi ? uint32_t((hi - kb_first + kWsKB - 1) / kWsKB) : 0;
  const uint32_t kt0 = uint32_t(kb_first / kWsKB);  // key tile of block 0

  if (warp == 1) tmem_alloc(&sh.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = sh.tmem_base;

  constexpr uint32_t id_o = idesc_tf32_bmn(kWsTQ, 64);
  // P V(j) of column group g: 4 k-steps x (P hi V hi, P hi V lo, P lo V hi)
  // into a fresh partial (keys 32 g .. 32 g + 31 of the block)
  auto issue_pv = [&](uint32_t j, uint32_t g) {
    const uint32_t ph = tm + 128 * (j % kWsIssuers), pl = ph + 64;
    const uint64_t dvh =
        smem_desc_sw128b32_mn(smem_addr(base + kWsOffV + (j & 1) * kWsSlot), kWsKRegion);
    const uint64_t dvl = dvh + (kWsTile >> 4);
#pragma unroll
    for (uint32_t kk = 0; kk < 4; ++kk) {
      const uint32_t ks = 4 * g + kk;
#pragma unroll
      for (uint32_t prod = 0; prod < 3; ++prod)
        mma_tf32_ts(tm + 384 + 64 * g, (prod == 2 ? pl : ph) + ks * 8,
                    (prod == 1 ? dvl : dvh) + ks * (1024 >> 4), id_o,
                    (kk > 0 || prod > 0) ? 1u : 0u);
    }
  };

  if (warp == 0) {
    // ---- V copies, and P V of column group 1 ----
    if (lane == 0) {
      // V of block j goes to slot j % 2 and completes on the full barrier of
      // its issuer j % 3 (each full barrier's waiters see its phases in order)
      uint32_t viss[kWsIssuers] = {0, 0, 0};
      auto load_v = [&](uint32_t j) {
        const uint32_t q = j % kWsIssuers;
        mbar_arrive_expect_tx(&sh.v_full[q], kWsSlot);
        bulk_load(base + kWsOffV + (j & 1) * kWsSlot,
                  vimg + (uint64_t(bh) * nkt + kt0 + j) * kWsSlot, kWsSlot, &sh.v_full[q]);
        ++viss[q];
      };
      for (uint32_t j = 0; j < 2 && j < nblk; ++j) load_v(j);
      for (uint32_t j = 0; j < nblk; ++j) {
        const uint32_t s = j & 1, q = j % kWsIssuers, use = j / kWsIssuers;
        // P V(j), group 1, beside the issuer's group 0
        if (!ws_wait(&sh.p_ready[q], use & 1, &sh) || !ws_wait(&sh.v_full[q], use & 1, &sh))
          break;
        tc_fence_after();
        issue_pv(j, 1);
        mma_commit(&sh.o_done[q]);
        mma_commit(&sh.v_empty[s]);
        // V(j + 2) once both halves of P V(j) have read slot s
        if (j + 2 < nblk) {
          if (!ws_wait(&sh.v_empty[s], (j >> 1) & 1, &sh)) break;
          load_v(j + 2);
        }
      }
      // every MMA this thread issued has completed, and the copies it issued
      // have landed, before the CTA can exit
      mma_commit(&sh.drain[kWsIssuers]);
      mbar_wait_bounded(&sh.drain[kWsIssuers], 0, kTcWait);
      mbar_wait_bounded(&sh.q_full, 0, kTcWait);
      for (uint32_t q = 0; q < kWsIssuers; ++q)
        if (viss[q] > 0) mbar_wait_bounded(&sh.v_full[q], (viss[q] - 1) & 1, kTcWait);
    }
    __syncwarp();
  } else if (warp <= kWsIssuers) {
    // ---- MMA issuer p: blocks j = p, p + 3, ... (S / P buffer p, K slot p, V slot j % 2) ----
    const uint32_t p = warp - 1;
    if (lane == 0 && nblk > p) {
      constexpr uint32_t id_s = idesc_tf32(kWsTQ, kWsKB);
      // descriptors built once; an offset moves the start address field
      // (address >> 4, no carry out of its 14 bits inside shared memory)
      const uint64_t dqh = smem_desc_sw128(smem_addr(qhi));
      const uint64_t dql = dqh + (kWsQPlane >> 4);
      const uint32_t ts = tm + 128 * p;
      // this issuer's K slot p: K(j) of its blocks, each loaded by the issuer
      // itself as soon as S of its previous block has read the slot
      uint8_t* kslot = base + kWsOffK + p * kWsSlot;
      const uint64_t dkh = smem_desc_sw128(smem_addr(kslot));
      const uint64_t dkl = dkh + (kWsTile >> 4);
      uint32_t kiss = 0;
      auto load_k = [&](uint32_t j) {
        mbar_arrive_expect_tx(&sh.k_full[p], kWsSlot);
        bulk_load(kslot, kimg + (uint64_t(bh) * nkt + kt0 + j) * kWsSlot, kWsSlot, &sh.k_full[p]);
        ++kiss;
      };
      load_k(p);
      bool ok = ws_wait(&sh.q_full, 0, &sh);
      for (uint32_t j = p; ok && j < nblk; j += kWsIssuers) {
        const uint32_t use = j / kWsIssuers, s = j & 1;
        // buffer p is free once both halves of P V(j - 3) have read P(j - 3)
        // (group 1 comes from the copy thread)
        if (use > 0 && !ws_wait(&sh.o_done[p], (use - 1) & 1, &sh)) break;
        if (!ws_wait(&sh.k_full[p], use & 1, &sh)) break;
        tc_fence_after();
        // S(j) = Q K^T: 8 k-steps x (hi hi, hi lo, lo hi)
#pragma unroll
        for (uint32_t ks = 0; ks < 8; ++ks) {
          const uint32_t oq = ((ks >> 2) * kWsQRegion + (ks & 3) * 32) >> 4;
          const uint32_t okk = ((ks >> 2) * kWsKRegion + (ks & 3) * 32) >> 4;
          mma_tf32_ss(ts, dqh + oq, dkh + okk, id_s, ks > 0);
          mma_tf32_ss(ts, dqh + oq, dkl + okk, id_s, 1);
          mma_tf32_ss(ts, dql + oq, dkh + okk, id_s, 1);
        }
        mma_commit(&sh.s_full[p]);
        mma_commit(&sh.k_empty[p]);
        // the next K of this issuer once these MMAs have read the slot (this
        // thread would wait for the softmax of block j now in any case)
        if (j + kWsIssuers < nblk) {
          if (!ws_wait(&sh.k_empty[p], use & 1, &sh)) break;
          load_k(j + kWsIssuers);
        }
        if (!ws_wait(&sh.p_ready[p], use & 1, &sh) || !ws_wait(&sh.v_full[p], use & 1, &sh))
          break;
        tc_fence_after();
        issue_pv(j, 0);  // group 1: the copy thread, at the same time
        mma_commit(&sh.o_done[p]);
        mma_commit(&sh.v_empty[s]);
      }
      // every MMA this thread issued has completed, and the copies it issued
      // have landed, before TMEM is freed and the CTA can exit
      mma_commit(&sh.drain[p]);
      mbar_wait_bounded(&sh.drain[p], 0, kTcWait);
      if (kiss > 0) mbar_wait_bounded(&sh.k_full[p], (kiss - 1) & 1, kTcWait);
    }
    __syncwarp();
  } else {
    // ---- softmax: thread = (query row, column group g of 32 keys) ----
    const uint32_t g = (warp - 1 - kWsIssuers) >> 2, quarter = warp & 3;
    const uint32_t row = quarter * 32 + lane;
    const uint32_t lane_off = (quarter * 32) << 16;
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
    float o[64];                    // this group's output row (f32 sum of the partials)
#pragma unroll
    for (int c = 0; c < 64; ++c) o[c] = 0.0f;
    bool inf_row = false, failed = false;
    uint32_t word_next = ~0u;  // mask word and summary byte of the next block
    uint8_t smy_next = 2;
    if (MASK && nblk > 0) {
      word_next = __ldg(wrow + kt0 * 256 + g * kWsTQ + row);
      smy_next = __ldg(srow + kt0);
    }
    // o = (o + the P V partial) * corr
    auto drain = [&](float corr) {
      const uint32_t tO = tm + 384 + 64 * g + lane_off;
#pragma unroll
      for (uint32_t c = 0; c < 64; c += 32) {
        float pv[32];
        tmem_ld16(tO + c, pv);
        tmem_ld16(tO + c + 16, pv + 16);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c + i] = __fmul_rn(__fadd_rn(o[c + i], pv[i]), corr);
      }
    };
    for (uint32_t j = 0; j < nblk; ++j) {
      const uint32_t p = j % kWsIssuers, ph = (j / kWsIssuers) & 1;
      const int64_t k0 = kb_first + int64_t(j) * kWsKB + 32 * g;  // key of column 0
      // this row's mask word of the block, loaded one block ahead
      uint32_t word = word_next;
      const uint8_t smy = smy_next;
      if (MASK && j + 1 < nblk) {
        word_next = __ldg(wrow + (kt0 + j + 1) * 256 + g * kWsTQ + row);
        smy_next = __ldg(srow + kt0 + j + 1);
      }
      if (!ws_wait_warp(&sh.s_full[p], ph, &sh)) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (smy & 2) word = ~0u;  // every (query, key) of the block kept
      {  // keys of the row's interval [r_lo, r_hi) as bits [c_lo, c_lo + c_span)
        const int64_t c_lo64 = max(int64_t(0), min(int64_t(32), r_lo - k0));
        const int64_t c_hi64 = max(c_lo64, min(int64_t(32), r_hi - k0));
        const uint32_t c_lo = uint32_t(c_lo64), c_span = uint32_t(c_hi64 - c_lo64);
        word &= c_span == 32 ? ~0u : c_span == 0 ? 0u : (((1u << c_span) - 1u) << c_lo);
      }
      const uint32_t tS = tm + 128 * p + 32 * g + lane_off;
      float sv[32];
      tmem_ld16(tS, sv);
      tmem_ld16(tS + 16, sv + 16);
      tmem_wait_ld();
      float mb = -INFINITY;
      if (!BIAS && word == ~0u) {  // every key of the block kept
#pragma unroll
        for (uint32_t c = 0; c < 32; ++c) {
          sv[c] = __fmul_rn(sv[c], a.scale);
          mb = fmaxf(mb, sv[c]);
        }
      } else {
#pragma unroll
        for (uint32_t c = 0; c < 32; ++c) {
          float sc = __fmul_rn(sv[c], a.scale);
          const bool kept = (word >> c) & 1;
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
      // (relative error ~2^-22), split into tf32 hi (over S) and lo
      const float mnl = mn == -INFINITY ? 0.0f : __fmul_rn(mn, kLog2e);
      float ps = 0.0f;
#pragma unroll
      for (uint32_t h = 0; h < 32; h += 16) {
        float phi[16], plo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float pr;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(pr) : "f"(__fmaf_rn(sv[h + i], kLog2e, -mnl)));
          ps = __fadd_rn(ps, pr);
          phi[i] = tf32_round_finite(pr);
          plo[i] = __fsub_rn(pr, phi[i]);
        }
        tmem_st16(tS + h, phi);
        tmem_st16(tS + 64 + h, plo);
      }
      l = __fmaf_rn(l, corr, ps);
      m = mn;
      // the partial of block j - 1 goes into o before P V(j) overwrites it
      // (P V(j) waits for this thread's p_ready). The parity wait on the
      // issuer of block j - 1 is exact: this thread waited for that issuer's
      // previous phase (block j - 4), and its next one (block j + 2) cannot
      // start before this thread's P(j + 2).
      if (j > 0) {
        const uint32_t q = (j - 1) % kWsIssuers;
        if (!ws_wait_warp(&sh.o_done[q], ((j - 1) / kWsIssuers) & 1, &sh)) {
          failed = true;
          break;
        }
        tc_fence_after();
        drain(corr);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sh.p_ready[p]);
    }
    if (!failed && nblk > 0) {  // the partial of the last block
      const uint32_t q = (nblk - 1) % kWsIssuers;
      failed = !ws_wait_warp(&sh.o_done[q], ((nblk - 1) / kWsIssuers) & 1, &sh);
      tc_fence_after();
      if (!failed) drain(1.0f);
    }
    if (!ws_softmax_any(failed)) {
      // merge the two column groups and write the output through shared
      // memory (the idle K and V rings): every thread leaves its row of O_g
      // and m_g, l_g there; then the 256 threads take 16-byte output chunks
      // in a rolled loop (code that runs once per CTA stays small)
      float* xo = reinterpret_cast<float*>(base + kWsOffK);  // [group][row][kWsStage]
      float* xs = xo + 2 * kWsTQ * kWsStage;                 // m, l: [group][row]
      int* xi = reinterpret_cast<int*>(xs + 4 * kWsTQ);      // +inf seen: [group][row]
#pragma unroll
      for (uint32_t c = 0; c < 64; c += 4)
        *reinterpret_cast<float4*>(xo + (g * kWsTQ + row) * kWsStage + c) =
            make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
      xs[g * kWsTQ + row] = m;
      xs[2 * kWsTQ + g * kWsTQ + row] = l;
      xi[g * kWsTQ + row] = inf_row;
      ws_softmax_sync();
      // per-row factors, once per row: O = (O_0 f0 + O_1 f1) / l
      float* xf = xs + 4 * kWsTQ + 2 * kWsTQ;  // past xi: [row][4] = f0, f1, 1 / l, empty
      if (g == 0) {
        const float m1 = xs[kWsTQ + row], l1 = xs[3 * kWsTQ + row];
        const float mx = fmaxf(m, m1);
        const float f0 = m == -INFINITY ? 0.0f : expf(m - mx);
        const float f1 = m1 == -INFINITY ? 0.0f : expf(m1 - mx);
        const float lsum = __fadd_rn(__fmul_rn(l, f0), __fmul_rn(l1, f1));
        const bool empty = nblk == 0 || lsum == 0.0f || inf_row || xi[kWsTQ + row] != 0;
        *reinterpret_cast<float4*>(xf + 4 * row) =
            make_float4(f0, f1, __frcp_rn(lsum), empty ? 1.0f : 0.0f);
      }
      ws_softmax_sync();
      const bool vec = a.out_feat == 1 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 &&
                       a.out_tok % 4 == 0 && a.out_batch % 4 == 0 &&
                       (!a.gate || ((reinterpret_cast<uintptr_t>(a.gate) & 15) == 0 &&
                                    a.gate_offset % 4 == 0));
      const float ev = a.empty_nan ? NAN : 0.0f;
#pragma unroll 1
      for (uint32_t idx = tid - 32 * (1 + kWsIssuers); idx < kWsTQ * 16; idx += 256) {
        const uint32_t r = idx >> 4, c4 = (idx & 15) * 4, qr = q0 + r;
        if (qr >= L) continue;
        const float4 fr = *reinterpret_cast<const float4*>(xf + 4 * r);
        const float f0 = fr.x, f1 = fr.y, rl = fr.z;
        const bool empty = fr.w != 0.0f;
        const float4 o0 = *reinterpret_cast<const float4*>(xo + r * kWsStage + c4);
        const float4 o1 = *reinterpret_cast<const float4*>(xo + (kWsTQ + r) * kWsStage + c4);
        auto mix = [&](float x0, float x1) {
          return empty ? ev : __fmul_rn(__fadd_rn(__fmul_rn(x0, f0), __fmul_rn(x1, f1)), rl);
        };
        float4 v4 = make_float4(mix(o0.x, o1.x), mix(o0.y, o1.y), mix(o0.z, o1.z), mix(o0.w, o1.w));
        if (vec) {
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
        } else {
          const uint64_t f = uint64_t(head) * 64 + c4;
          store_out(a, b, qr, f, v4.x);
          store_out(a, b, qr, f + 1, v4.y);
          store_out(a, b, qr, f + 2, v4.z);
          store_out(a, b, qr, f + 3, v4.w);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_free(tm, 512);
}
