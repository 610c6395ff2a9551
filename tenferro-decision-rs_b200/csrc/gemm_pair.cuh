// gemm_pair.cuh -- the GEMM-epilogue kernel on CTA pairs (tcgen05 cta_group::2;
// included by gemm_epilogue.cu inside its anonymous namespace, after the
// one-CTA kernel, whose GemmArgs, GemmShared, gemm_wait and epi_store it uses).
//
// A cluster of two CTAs on two SMs computes a 256-token x 256-output tile with
// one M256 N256 K8 MMA per k-step, issued by the even CTA (the leader): each CTA
// holds its 128 tokens of x (A) and half of the weight tile (B: the leader the
// output rows [0, 128) of the tile, the other CTA rows [128, 256)), and the
// tensor cores of each SM read the A rows they own and both B halves. So each
// SM's shared memory serves 8 KB per MMA instead of 12 KB on one CTA (extra
// shared-memory traffic slows the one-CTA kernel in proportion), and a stage
// is 64 KB, so three stages fit; measured 6 - 9 % faster than one CTA per
// tile. Each CTA's tensor memory holds the accumulator rows of its own tokens,
// which its own epilogue warps drain, exactly as on one CTA.
//
// Barriers: each CTA's producer loads its own halves and signals the leader's
// full barrier (expecting both CTAs' bytes); the leader's MMA commits the
// stage's empty barrier and the partials' full barriers in both CTAs (one
// commit to each CTA's barrier); the epilogue warps of both CTAs release a
// partial on the leader's empty barrier (16 arrivals). Every wait is bounded; a
// CTA that gives up stops its roles, and both CTAs meet at the cluster barrier
// at the end in any case. Every copy is a plain tiled load into the issuing
// CTA's own shared memory.

__device__ __forceinline__ uint32_t pair_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Whole warp, the same warp in both CTAs; the same dst offset in both.
__device__ __forceinline__ void pair_tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void pair_tmem_free(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void pair_mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc,
                                                 uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void pair_commit_own(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}
// Arrives once on `bar` (the same offset) in both CTAs when the MMAs this
// thread issued before have completed: a commit to each CTA's barrier.
__device__ __forceinline__ void pair_commit_both(uint64_t* bar) {
  pair_commit_own(bar);
  asm volatile(
      "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [ra];\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(1u)
      : "memory");
}
// Box (c0, c1) of `map` into this CTA's shared memory at dst; the bytes
// complete on the leader's barrier at the offset of `bar`.
__device__ __forceinline__ void pair_tma_load_2d(void* dst, const CUtensorMap* map,
                                                 uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1),
      "r"(smem_addr(bar) & 0xFEFFFFFFu)
      : "memory");
}
// Arrives on the leader's barrier at the offset of `bar`.
__device__ __forceinline__ void pair_arrive_leader(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_addr(bar)),
      "r"(0u)
      : "memory");
}

// The pair's next piece of work from item i (advanced past it); false at the
// end. Pair tile rows are 256 tokens (two 128-token tiles). Non-batched and
// batched calls without a causal schedule: pair tiles dealt round robin;
// kCausalOut (batch_tokens == nout): pair row r of a batch needs the 256-wide
// output tiles n <= r, numbered as a triangle; kCausalK (in_dim ==
// batch_tokens): pair row r contracts over 256 (r + 1) keys, in chunks of 256
// keys (8 stages) split evenly over the pairs (a.split, row_tokens 256).
__device__ __forceinline__ bool next_pair_piece(const GemmArgs& a, uint32_t nst, uint32_t pair,
                                                uint32_t npairs, uint64_t& i, GemmPiece& p) {
  constexpr uint32_t kChunkStages = 8;  // 256 keys of 32
  if (a.causal == kCausalK) {
    const uint64_t end = a.split.start(pair + 1);
    if (i >= end) return false;
    const uint32_t batch = uint32_t(i / a.split.per_batch);
    const uint64_t r = i - uint64_t(batch) * a.split.per_batch;
    const uint32_t pr = CausalKSplit::row_of(r);
    const uint32_t c0 = uint32_t(r - CausalKSplit::prefix(pr));
    const uint32_t c1 = uint32_t(min(uint64_t(pr) + 1, uint64_t(c0) + (end - i)));
    p.m = batch * a.split.mb + pr;  // pair row
    p.n = 0;
    p.s0 = c0 * kChunkStages;
    p.s1 = min(nst, c1 * kChunkStages);
    p.slot = pair - a.split.owner(a.split.first(batch, pr));
    p.skip = false;
    i += c1 - c0;
    return true;
  }
  if (i >= a.items) return false;
  if (a.causal == kCausalOut) {
    const uint32_t rows = a.mb / 2;  // pair rows per batch
    const uint64_t per = CausalKSplit::prefix(rows);
    const uint32_t batch = uint32_t(i / per);
    const uint64_t r = i - uint64_t(batch) * per;
    const uint32_t pr = CausalKSplit::row_of(r);
    p.m = batch * rows + pr;
    p.n = uint32_t(r - CausalKSplit::prefix(pr));
  } else {
    p.m = uint32_t(i / a.ntiles);
    p.n = uint32_t(i - uint64_t(p.m) * a.ntiles);
  }
  p.s0 = 0;
  p.s1 = nst;
  p.slot = 0;
  p.skip = false;
  i += npairs;
  return true;
}

// Tiles with non-finite operands are computed here too and then overwritten by
// the SIMT kernel (calls with pre-split operands have none).
// FK: K values per partial (32 or 64: one or two stages between drains).
template <int EPI, int ACT, bool BIAS, int FK>
__global__ void __launch_bounds__(kGThreads, 1) gemm_pair_tc_kernel(
    const __grid_constant__ CUtensorMap xh_map, const __grid_constant__ CUtensorMap xl_map,
    const __grid_constant__ CUtensorMap wh_map, const __grid_constant__ CUtensorMap wl_map,
    GemmArgs a) {
  constexpr int SK = 32;
  constexpr int kStages = 3;
  constexpr uint32_t kABytes = kBM * SK * 4;             // 128 tokens x 32 (16 KB)
  constexpr uint32_t kBHalf = (kBN / 2) * SK * 4;        // 128 output rows x 32 (16 KB)
  constexpr uint32_t kStageBytes = 2 * kABytes + 2 * kBHalf;  // 64 KB
  static_assert(kStages * kStageBytes + 1024 <= kGemmSmem, "stage ring");
  static_assert(kGemmSmemAll <= 227 * 1024, "stage ring + staging tiles");
  constexpr uint32_t kSpf = FK / SK;  // stages per partial
  static_assert(FK % SK == 0, "partial length");
  const uint32_t nst = a.nk;  // K chunks of 32
  extern __shared__ __align__(1024) uint8_t gemm_smem[];
  __shared__ GemmShared sh;
  pdl_enter();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = pair_rank();
  const uint32_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) &
                                             ~uintptr_t(1023));
  const uint64_t first = a.causal == kCausalK ? a.split.start(pair) : uint64_t(pair);

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);   // the leader's expect-tx arrival (+ both CTAs' bytes)
      mbar_init(&sh.empty[s], 1);  // the leader's MMA commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.part_full[b], 1);
      mbar_init(&sh.part_empty[b], 2 * kEpiWarps);  // both CTAs' epilogue warps
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    mbar_init_fence();
  }
  if (warp == 1) pair_tmem_alloc(&sh.tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  pair_sync();  // both CTAs' barriers exist before either signals the other's
  tc_fence_after();
  const uint32_t tm = sh.tmem_base;

  if (warp == 0) {
    // ---- TMA producer (both CTAs): this CTA's x rows and weight half ----
    if (lane == 0) {
      uint32_t g = 0;
      bool ok = true;
      uint64_t it = first;
      GemmPiece pc;
      while (ok && next_pair_piece(a, nst, pair, npairs, it, pc)) {
        const uint32_t pm = pc.m, n = pc.n;
        const int row_x = int((2 * pm + rank) * kBM);
        const int row_w = EPI == kEpiGeglu
                              ? int(rank * a.inter + n * (kBN / 2))
                              : int(batch_wrow(a, 2 * pm * kBM) + n * kBN + rank * (kBN / 2));
        for (uint32_t kc = pc.s0; kc < pc.s1; ++kc, ++g) {
          const uint32_t s = g % kStages, use = g / kStages;
          if (use > 0 && !gemm_wait(&sh.empty[s], (use - 1) & 1, &sh)) {
            ok = false;
            break;
          }
          uint8_t* st = base + size_t(s) * kStageBytes;
          if (rank == 0) mbar_arrive_expect_tx(&sh.full[s], 2 * kStageBytes);
          const int k = int(kc * SK);
          pair_tma_load_2d(st, &xh_map, &sh.full[s], k, row_x);
          pair_tma_load_2d(st + kABytes, &xl_map, &sh.full[s], k, row_x);
          pair_tma_load_2d(st + 2 * kABytes, &wh_map, &sh.full[s], k, row_w);
          pair_tma_load_2d(st + 2 * kABytes + kBHalf, &wl_map, &sh.full[s], k, row_w);
        }
      }
      // the MMAs have read (so the copies have landed in) every stage issued
      for (uint32_t s = 0; s < kStages && s < g; ++s) {
        const uint32_t uses = (g - 1 - s) / kStages + 1;  // uses of stage s
        mbar_wait_bounded(&sh.empty[s], (uses - 1) & 1, kGemmWait);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: the leader's thread 0 ----
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(2 * kBM, kBN);
      uint32_t g = 0, pg = 0;
      bool ok = true;
      uint64_t it = first;
      GemmPiece pc;
      while (ok && next_pair_piece(a, nst, pair, npairs, it, pc)) {
        for (uint32_t kc = pc.s0; kc < pc.s1; ++kc, ++g) {
          const uint32_t s = g % kStages, use = g / kStages;
          const uint32_t pb = pg & 1, puse = pg >> 1;
          const bool first = (kc - pc.s0) % kSpf == 0;
          if ((first && puse > 0 && !gemm_wait(&sh.part_empty[pb], (puse - 1) & 1, &sh)) ||
              !gemm_wait(&sh.full[s], use & 1, &sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tm + pb * kBN;
          const uint32_t st = smem_addr(base + size_t(s) * kStageBytes);
          const uint32_t ah = st, al = st + kABytes, bh = st + 2 * kABytes, bl = bh + kBHalf;
#pragma unroll
          for (uint32_t ks = 0; ks < SK / 8; ++ks)  // x hi * w lo (starts the partial)
            pair_mma_tf32_ss(d, smem_desc_sw128(ah + ks * 32), smem_desc_sw128(bl + ks * 32),
                             idesc, !first || ks != 0);
#pragma unroll
          for (uint32_t ks = 0; ks < SK / 8; ++ks)  // x lo * w hi
            pair_mma_tf32_ss(d, smem_desc_sw128(al + ks * 32), smem_desc_sw128(bh + ks * 32),
                             idesc, 1);
#pragma unroll
          for (uint32_t ks = 0; ks < SK / 8; ++ks)  // x hi * w hi
            pair_mma_tf32_ss(d, smem_desc_sw128(ah + ks * 32), smem_desc_sw128(bh + ks * 32),
                             idesc, 1);
          pair_commit_both(&sh.empty[s]);
          if ((kc - pc.s0) % kSpf == kSpf - 1 || kc + 1 == pc.s1) {
            pair_commit_both(&sh.part_full[pb]);
            ++pg;
          }
        }
      }
      pair_commit_own(&sh.drain);
      mbar_wait_bounded(&sh.drain, 0, kGemmWait);
    }
    __syncwarp();
  } else {
    // ---- epilogue (both CTAs): this CTA's 128 tokens of the pair tile ----
    const uint32_t q = warp & 3;
    const uint32_t half = (warp - 2) >> 2;
    const uint32_t row = q * 32 + lane;
    const uint32_t lane_off = (q * 32) << 16;
    const uint32_t c_lo = EPI == kEpiGeglu ? 64 * half : 128 * half;
    const uint32_t c_hi = EPI == kEpiGeglu ? 128 + 64 * half : 128 * half + 64;
    float2 acc2[64];
    uint32_t g = 0;
    bool ok = true;
    uint64_t it = first;
    GemmPiece pc;
    while (ok && next_pair_piece(a, nst, pair, npairs, it, pc)) {
      const uint32_t pm = pc.m, n = pc.n;
      const uint32_t tpart = (pc.s1 - pc.s0 + kSpf - 1) / kSpf;
#pragma unroll
      for (int j = 0; j < 64; ++j) acc2[j] = make_float2(0.0f, 0.0f);
      for (uint32_t kc = 0; kc < tpart; ++kc, ++g) {
        const uint32_t pb = g & 1, puse = g >> 1;
        bool got = true;
        if (lane == 0) got = gemm_wait(&sh.part_full[pb], puse & 1, &sh);
        if (!__shfl_sync(0xffffffffu, int(got), 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t src = tm + pb * kBN + lane_off;
#pragma unroll
        for (int c = 0; c < 128; c += 16) {
          float v[16];
          tmem_ld16(src + (c < 64 ? c_lo + c : c_hi + c - 64), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j += 2)
            acc2[(c + j) / 2] = __fadd2_rn(acc2[(c + j) / 2], make_float2(v[j], v[j + 1]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) pair_arrive_leader(&sh.part_empty[pb]);
      }
      if (!ok) break;
      if constexpr (EPI == kEpiBiasAct && ACT == TFX_ACT_IDENTITY && !BIAS) {
        if (a.stage_rows) {  // the whole warp, rows past the length included
          const uint32_t o0 = n * kBN + 128 * half;
          if (o0 < a.nout)
            epi_store_staged(a, (2 * pm + rank) * kBM + q * 32, lane, o0, pc.slot,
                             reinterpret_cast<const float*>(acc2),
                             reinterpret_cast<float*>(base + size_t(kStages) * kStageBytes) +
                                 (warp - 2) * 1024);
          continue;
        }
      }
      const uint32_t t = (2 * pm + rank) * kBM + row;
      if (t >= a.length) continue;
      epi_store<EPI, ACT, BIAS>(a, t, n, half, pc.slot, reinterpret_cast<float*>(acc2));
    }
  }
  tc_fence_before();
  __syncthreads();
  pair_sync();  // every signal between the CTAs has landed; the leader's MMAs are done
  tc_fence_after();
  if (warp == 1) pair_tmem_free(tm, 512);
}
