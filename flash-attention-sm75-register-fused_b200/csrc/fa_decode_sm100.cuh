// Decode attention for B200 (sm_100a): query blocks of at most 16 rows per
// (batch, KV head) -- one token per query head of a GQA group, or a few
// tokens of a short chunk -- against a long K/V cache.  Included by
// fa_fwd_sm100.cu, whose helpers (bounded mbarrier waits, the device status
// word, pack2, kv_tiles_core) it uses.
//
// The same online softmax as the attention kernel (running max m, sum l, O
// rescaled when m grows; flash-attention-sm75-fused/include/online_step.cuh:
// 36-126), arranged for few query rows: keys lie on the MMA's M dimension.
//
//   S^T = K_j Q^T        M = 128 keys (one TMEM lane each), N = 16 query rows
//   P   = exp2(S - m)    written by the key's thread into shared memory as
//                        the K-major B operand [16 rows x 128 keys] (4 KB,
//                        double-buffered)
//   O^T += V_j^T P^T     M = d (one TMEM lane per column of O; d = 64 pads M
//                        to 128 with rows that are never read), N = 16
//
// so each thread computes R <= 16 exponentials per 128-key tile (R = the
// block's rows rounded up to 4, 8 or 16) instead of 128, S^T is
// double-buffered in TMEM (the scores of tile j+1 are computed while the
// softmax of tile j runs), and the tensor core reads only K, V and the small
// Q and P operands from shared memory.  The rows' maxima are combined across
// the four softmax warps once per tile (named barrier with an AND of the
// warps' status, so a failed wait makes all four leave together).
//
// Work items are (batch*head, key split) pairs walked by persistent CTAs; the
// K/V ring and the Q double buffer carry over from one item to the next.  A
// split writes a normalised partial O and its LSE for fa_combine_kernel
// (n_splits > 1), otherwise the final O / LSE.
//
// Warps: 0-3 softmax (thread t = key t of the tile, and column t of O^T for
// its rescale and the epilogue; 8-row blocks: warps 0-7 and 16-row blocks:
// warps 0-15, warp w + 4k taking the k-th share of the rows of the same
// keys), then the TMA producer and the MMA issuer + TMEM owner (192, 320 or
// 576 threads).
//
// Development builds (-DFA_TRACE) record per tile c of the CTA (c < 63):
// producer issued K_c / V_c (0, 1); MMA warp issued S^T(c) / PV(c) (2, 3),
// saw K_c / V_c land (8, 9) and P(c) (10); softmax warp 0 saw S^T(c) (4),
// passed the tile's barrier (5), arrived on P(c) (6), saw PV(c-2) done (7);
// row 63: CTA set up / done (30, 31).
namespace fa {
namespace {


// critical-path waits poll (bar_wait_spin) instead of suspending
#ifndef FA_DEC_SPIN
#define FA_DEC_SPIN 1
#endif
__device__ __forceinline__ bool dec_wait(uint32_t bar, uint32_t parity, const WaitCtl& c, int site) {
#if FA_DEC_SPIN
  return bar_wait_spin(bar, parity, c, site);
#else
  return bar_wait(bar, parity, c, site);
#endif
}
constexpr int kDecRows = 16;  // query rows per item: the S^T MMA's N

template <int D>
struct DecLayout {
  // keys per K/V tile (a softmax round): 256 at d = 64, so that every tile
  // carries 32 KB and the per-round chain is paid per 32 KB; a thread then
  // owns keys t and t + 128 (two "halves")
  static constexpr int kKeys = (D == 64) ? 256 : 128;
  static constexpr int kHalves = kKeys / 128;
  static constexpr int kTile = kKeys * D * 2;            // one K or V tile (32 KB)
  static constexpr int kBlockBytes = kKeys * 128;        // 64-column block of a tile
  static constexpr int kSlots = 6;                       // K/V ring (192 KB)
  static constexpr int kQBytes = kDecRows * D * 2;       // 16-row Q block
  static constexpr int kQBlock = kDecRows * 128;         // 64-column block of it
  // P buffer b: kKeys / 64 blocks of [16 rows x 128 B] at kOffP + b * kPBuf
  static constexpr int kPRows = kDecRows * 128;          // 2 KB
  static constexpr int kPBuf = (kKeys / 64) * kPRows;
  // shared memory (offsets from a 1024-aligned base).  At d = 64 the PV's
  // unused M rows 64-127 read 16 KB past each K step's V rows, up to 48 KB
  // past a slot's start: for the last slot that is the P buffers, so the ring
  // comes first and P right after it.
  static constexpr int kOffKV = 0;
  static constexpr int kOffP = kOffKV + kSlots * kTile;
  static constexpr int kOffQ = kOffP + 2 * kPBuf;  // Q double buffer
  static constexpr int kOffRed = kOffQ + 2 * kQBytes;    // [2][4 warps][16] row maxima
  static constexpr int kOffSum = kOffRed + 2 * 4 * kDecRows * 4;  // [4 warps][16] row sums
  static constexpr int kOffBar = kOffSum + 4 * kDecRows * 4;
  // named barrier of the four softmax warps
  static constexpr uint32_t kNamedBar = 1;
  // barriers
  static constexpr int kBarQ = 0;                        // 2 (TMA)
  static constexpr int kBarQFree = 2;                    // 2 (MMA commit)
  static constexpr int kBarFull = 4;                     // kSlots (TMA)
  static constexpr int kBarEmpty = kBarFull + kSlots;    // kSlots (MMA commit)
  static constexpr int kBarS = kBarEmpty + kSlots;       // 2 (MMA commit): S^T buffer written
  static constexpr int kBarSFree = kBarS + 2;            // 2 (128 arrivals): S^T buffer read
  static constexpr int kBarP = kBarSFree + 2;            // 2 (128 arrivals): P buffer written
  static constexpr int kBarPV = kBarP + 2;               // 2 (MMA commit): PV from P buffer done
  static constexpr int kBarOFree = kBarPV + 2;           // 1 (128 arrivals): epilogue read O
  static constexpr int kBarDrain = kBarOFree + 1;        // 1 (MMA commit)
  static constexpr int kNumBars = kBarDrain + 1;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kDynBytes = kBytes + 1024;
  // tensor memory: S^T buffer b at columns 16 * kHalves * b (16 columns per
  // half), O^T after them
  static constexpr uint32_t kTmemCols = 32 * kHalves * 2;
  __host__ __device__ static constexpr uint32_t tS(int b) { return b ? 16u * kHalves : 0u; }
  static constexpr uint32_t tO = 32 * kHalves;
  static_assert(kDynBytes <= 227 * 1024, "shared memory budget");
  static_assert(D == 128 || kOffKV + (kSlots - 1) * kTile + 16384 + kKeys * 128 <= kOffQ,
                "d = 64: the V^T operand's padding rows stay inside the ring and P");
  static_assert(kOffKV % 1024 == 0 && kOffQ % 1024 == 0 && kTile % 1024 == 0 &&
                    kQBytes % 1024 == 0 && kPBuf % 1024 == 0 && kOffP % 1024 == 0,
                "128-byte-swizzled operands need 1024-byte alignment");
};

struct DecItem {
  int bh, sp, bh_kv;
  int jb, n;  // first K/V tile and tile count of the split
};

__device__ __forceinline__ void dec_item(const FwdParams& p, int w, DecItem& it) {
  it.sp = w % p.n_splits;
  it.bh = w / p.n_splits;
  const int b = it.bh / p.heads;
  it.bh_kv = b * p.Hkv + (it.bh % p.heads) / p.group;
  // all rows are in query tile 0
  const int total = kv_tiles_for_tile(p, 0);
  it.jb = it.sp * p.tiles_per_split;
  it.n = max(0, min(total, it.jb + p.tiles_per_split) - it.jb);
}

// Transposed butterfly over the warp: v[R] per lane in; out, the reduction
// over all 32 lanes of row dec_row<R>(lane) (lanes with the low lane bits
// dec_low<R>() clear hold it).  log2(R) halving steps on lane bits 16, 8, ..
// then a plain butterfly over the remaining bits.
template <int R>
__device__ __forceinline__ constexpr int dec_low() {
  return (16 >> (R == 4 ? 2 : R == 8 ? 3 : 4)) * 2 - 1;
}
template <int R, bool kMax>
__device__ __forceinline__ float dec_reduce(float (&v)[R], int lane) {
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
  constexpr int kSteps = R == 4 ? 2 : R == 8 ? 3 : 4;
#pragma unroll
  for (int step = 0; step < kSteps; ++step) {
    // rows [0, 2*half) -> [0, half): lanes with lane bit `bit` set keep the
    // upper half of the rows, their partners the lower half
    const int half = (R / 2) >> step;
    const int bit = 16 >> step;
    const bool hi = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = hi ? v[i] : v[i + half];
      const float keep = hi ? v[i + half] : v[i];
      v[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, bit));
    }
  }
  float r = v[0];
#pragma unroll
  for (int bit = 16 >> kSteps; bit >= 1; bit >>= 1) r = op(r, __shfl_xor_sync(0xffffffffu, r, bit));
  return r;
}

template <int R>
__device__ __forceinline__ int dec_row(int lane) {
  constexpr int kSteps = R == 4 ? 2 : R == 8 ? 3 : 4;
  int row = 0;
#pragma unroll
  for (int step = 0; step < kSteps; ++step)
    if (lane & (16 >> step)) row += (R / 2) >> step;
  return row;
}

// RS = 2 or 4 splits a block's rows between that many softmax warpgroups
// (warps w, w + 4, ... read the same TMEM lanes, i.e. the same keys, and
// different row columns), dividing each thread's exponentials by RS.
template <int D, bool BF16, int R, int RS>
__global__ void __launch_bounds__(32 * (4 * RS + 2), 1) fa_decode_kernel(const __grid_constant__ FwdParams p) {
  static_assert(R == 4 || R == 8 || R == 16, "rows per block");
  static_assert(RS == 1 || (RS == 2 && R >= 8) || (RS == 4 && R == 16), "row split");
  constexpr int kDecWarpLoad = 4 * RS;
  constexpr int kDecWarpMma = 4 * RS + 1;
  constexpr uint32_t kSoftThreads = 128 * RS;
  using L = DecLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };
  const int n_work = p.B * p.heads * p.n_splits;

  // ---- set-up
  if (threadIdx.x == 0) {
    const unsigned long long st = *reinterpret_cast<volatile unsigned long long*>(&g_fa_status);
    *abort_flag = ((st >> 32) == p.epoch && (st & 0xffffffffull) != 0ull) ? 1 : 0;
    for (int i = 0; i < L::kNumBars; ++i) {
      const bool all = (i == L::kBarSFree || i == L::kBarSFree + 1 || i == L::kBarP ||
                        i == L::kBarP + 1 || i == L::kBarOFree);
      ptx::mbar_init(bar(i), all ? kSoftThreads : 1u);
    }
    ptx::fence_barrier_init();
  }
  // P rows past the block (R..15) are never written: zero them once
  if (warp < 4 * RS) {
    uint4* pz = reinterpret_cast<uint4*>(smem + L::kOffP);
    for (int i = threadIdx.x; i < 2 * L::kPBuf / 16; i += kSoftThreads) pz[i] = make_uint4(0u, 0u, 0u, 0u);
    ptx::fence_proxy_async_smem();
  }
  __syncthreads();
  if (*abort_flag) return;
  if (warp == kDecWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), L::kTmemCols);
    ptx::tmem_relinquish();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};
  if (threadIdx.x == 0) FA_TRACE_AT(kTraceTiles - 1, 30);
  // the split combine (a programmatic dependent) may launch now; it waits
  // for this grid's completion before it reads anything
  ptx::launch_dependents();

  if (warp == kDecWarpLoad) {
    // ===================================================== TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&p.tm_q);
      ptx::prefetch_tmap(&p.tm_k);
      ptx::prefetch_tmap(&p.tm_v);
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_first();  // each K/V tile is read once
      int ring = 0, k = 0, q_loads[2] = {0, 0};
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_work; w += gridDim.x) {
        DecItem it;
        dec_item(p, w, it);
        if (it.n == 0) continue;
        const int qb = k & 1;
        // item k's Q overwrites the buffer of item k-2, once its S MMAs completed
        if (k >= 2 && !(ok = bar_wait(bar(L::kBarQFree + qb), ((k - 2) >> 1) & 1, wc, 40))) break;
        ptx::mbar_arrive_expect_tx(bar(L::kBarQ + qb), L::kQBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          ptx::tma_load_3d(sbase + L::kOffQ + qb * L::kQBytes + c * L::kQBlock, &p.tm_q,
                           bar(L::kBarQ + qb), c * 64, 0, it.bh, pol_q);
        ++q_loads[qb];
        const int nr = (it.n + L::kHalves - 1) / L::kHalves;  // rounds of kKeys keys
        for (int i = 0; i < 2 * nr; ++i, ++ring) {  // K_j, V_j, K_j+1, ...
          const int slot = ring % L::kSlots;
          if (ring >= L::kSlots &&
              !(ok = dec_wait(bar(L::kBarEmpty + slot), ((ring / L::kSlots) - 1) & 1, wc, 41)))
            break;
          const void* map = (i & 1) ? static_cast<const void*>(&p.tm_v)
                                    : static_cast<const void*>(&p.tm_k);
          const uint32_t dst = sbase + L::kOffKV + slot * L::kTile;
          ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            ptx::tma_load_3d(dst + c * L::kBlockBytes, map, bar(L::kBarFull + slot), c * 64,
                             (it.jb + (i >> 1) * L::kHalves) * kBlockN, it.bh_kv, pol_kv);
          FA_TRACE_AT(ring >> 1, ring & 1);
        }
        ++k;
      }
      // every copy this thread started lands before the CTA exits
      for (int r = max(0, ring - L::kSlots); r < ring; ++r)
        bar_wait(bar(L::kBarFull + r % L::kSlots), (r / L::kSlots) & 1, wc, 42, false);
      for (int b = 0; b < 2; ++b)
        if (q_loads[b] > 0) bar_wait(bar(L::kBarQ + b), (q_loads[b] - 1) & 1, wc, 42, false);
    }
  } else if (warp == kDecWarpMma) {
    // ===================================================== MMA issuer
    constexpr uint32_t fmt = BF16 ? 1u : 0u;
    constexpr uint32_t idesc_s = ptx::make_idesc_f16(kBlockN, kDecRows, fmt, 0, 0);
    constexpr uint32_t idesc_pv = ptx::make_idesc_f16(128, kDecRows, fmt, 1, 0);
    const uint64_t k_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, 16, 1024);
    const uint64_t v_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, 16384, 1024);
    const uint64_t q_desc0 = ptx::smem_desc_sw128(sbase + L::kOffQ, 16, 1024);
    const uint64_t p_desc = ptx::smem_desc_sw128(sbase + L::kOffP, 16, 1024);
    // V as the MN-major A operand of O^T: M = d in 64-row blocks 16 KB apart
    // (d = 128: the tile's second column block, the same descriptor as V in
    // the attention kernel's PV; d = 64: rows 64-127 of M read the tile's
    // second half, products that land in O^T lanes that are never read)
    auto slot_of = [](int item) { return item % L::kSlots; };
    auto phase_of = [](int item) { return static_cast<uint32_t>((item / L::kSlots) & 1); };
    auto wait = [&](uint32_t b, uint32_t ph, int site) {
      return __all_sync(0xffffffffu, dec_wait(b, ph, wc, site));
    };
    // S^T(c) = K_c Q^T into buffer c & 1 (K = ring item 2c, Q buffer qb)
    auto issue_s = [&](int c, int qb, bool last_of_item) -> bool {
      if (!wait(bar(L::kBarFull + slot_of(2 * c)), phase_of(2 * c), 43)) return false;
      if (lane == 0) FA_TRACE_AT(c, 8);
      if (c >= 2 && !wait(bar(L::kBarSFree + (c & 1)), ((c >> 1) - 1) & 1, 44)) return false;
      ptx::tc_fence_after();
      if (lane == 0) FA_TRACE_AT(c, 2);
      const uint64_t kd = k_desc0 + static_cast<uint64_t>((slot_of(2 * c) * L::kTile) >> 4);
      const uint64_t qd = q_desc0 + static_cast<uint64_t>((qb * L::kQBytes) >> 4);
      if (ptx::elect_one()) {
        // half h: keys 128h.. of the tile (rows 16 KB further) into 16 columns
#pragma unroll
        for (int h = 0; h < L::kHalves; ++h)
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            ptx::mma_ss(tmem + L::tS(c & 1) + 16 * h,
                        kd + static_cast<uint64_t>(
                                 (h * 16384 + (kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4),
                        qd + static_cast<uint64_t>(((kk / 4) * L::kQBlock + (kk % 4) * 32) >> 4),
                        idesc_s, kk > 0 ? 1u : 0u);
        ptx::mma_commit(bar(L::kBarS + (c & 1)));
        ptx::mma_commit(bar(L::kBarEmpty + slot_of(2 * c)));
        if (last_of_item) ptx::mma_commit(bar(L::kBarQFree + qb));
      }
      __syncwarp();
      return true;
    };
    // O^T (+)= V_c^T P^T (P buffer c & 1, V = ring item 2c+1); the first tile
    // of item k starts the accumulator once the epilogue of item k-1 read it
    auto issue_pv = [&](int c, bool first, int k) -> bool {
      if (!wait(bar(L::kBarP + (c & 1)), (c >> 1) & 1, 45)) return false;
      if (lane == 0) FA_TRACE_AT(c, 10);
      if (!wait(bar(L::kBarFull + slot_of(2 * c + 1)), phase_of(2 * c + 1), 46)) return false;
      if (lane == 0) FA_TRACE_AT(c, 9);
      if (first && k > 0 && !wait(bar(L::kBarOFree), (k - 1) & 1, 47)) return false;
      ptx::tc_fence_after();
      if (lane == 0) FA_TRACE_AT(c, 3);
      const uint64_t vd = v_desc0 + static_cast<uint64_t>((slot_of(2 * c + 1) * L::kTile) >> 4);
      const uint64_t pd = p_desc + static_cast<uint64_t>(((c & 1) * L::kPBuf) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < L::kKeys / 16; ++kk)
          ptx::mma_ss(tmem + L::tO, vd + static_cast<uint64_t>((kk * 2048) >> 4),
                      pd + static_cast<uint64_t>(((kk / 4) * L::kPRows + (kk % 4) * 32) >> 4),
                      idesc_pv, (first && kk == 0) ? 0u : 1u);
        ptx::mma_commit(bar(L::kBarPV + (c & 1)));
        ptx::mma_commit(bar(L::kBarEmpty + slot_of(2 * c + 1)));
      }
      __syncwarp();
      return true;
    };
    // Issue order: S^T(c) and PV(c-1), the PV first when K_c has not landed
    // yet (the softmax of tile c cannot start before it anyway).
    bool ok = true;
    int c = 0, k = 0;
    bool pending = false;
    int pend_c = 0, pend_k = 0;
    bool pend_first = false;
    for (int w = blockIdx.x; ok && w < n_work; w += gridDim.x) {
      DecItem it;
      dec_item(p, w, it);
      if (it.n == 0) continue;
      const int qb = k & 1;
      const int nr = (it.n + L::kHalves - 1) / L::kHalves;
      for (int j = 0; ok && j < nr; ++j, ++c) {
        if (pending && !ptx::mbar_test_wait(bar(L::kBarFull + slot_of(2 * c)), phase_of(2 * c))) {
          if (!(ok = issue_pv(pend_c, pend_first, pend_k))) break;
          pending = false;
        }
        if (j == 0 && !(ok = wait(bar(L::kBarQ + qb), (k >> 1) & 1, 48))) break;
        if (!(ok = issue_s(c, qb, j == nr - 1))) break;
        if (pending && !(ok = issue_pv(pend_c, pend_first, pend_k))) break;
        pending = true;
        pend_c = c;
        pend_k = k;
        pend_first = j == 0;
      }
      ++k;
    }
    if (ok && pending) issue_pv(pend_c, pend_first, pend_k);
    // all MMAs complete before TMEM is released
    if (ptx::elect_one()) ptx::mma_commit(bar(L::kBarDrain));
    __syncwarp();
    bar_wait(bar(L::kBarDrain), 0, wc, 49, false);
  } else {
    // ===================================================== softmax (warps 0 .. 4 RS - 1)
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    const int t = threadIdx.x & 127;  // key of the tile (and t + 128: half 1), TMEM lane
    constexpr int H = L::kHalves;
    constexpr int RP = R / RS;        // rows of this thread: q0 .. q0 + RP - 1
    const int q0 = (warp >> 2) * RP;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    // this thread's RP row columns starting at TMEM column `col` (+ q0)
    auto ld_rows = [&](uint32_t col, uint32_t (&r)[16]) {
      if constexpr (RP == 16) ptx::tmem_ld16(tmem + lane_base + col, r);
      else if constexpr (RP == 8) ptx::tmem_ld8(tmem + lane_base + col + q0, r);
      else ptx::tmem_ld4(tmem + lane_base + col + q0, r);
    };
    // (stores exactly this thread's RP columns: other warpgroups own the rest)
    auto st_rows = [&](uint32_t col, const uint32_t (&r)[16]) {
      if constexpr (RP == 16) ptx::tmem_st16(tmem + lane_base + col, r);
      else if constexpr (RP == 8) ptx::tmem_st8(tmem + lane_base + col + q0, r);
      else ptx::tmem_st4(tmem + lane_base + col + q0, r);
    };
    const int nrows = p.Nq;
    // keys below vis_all are visible to every row of the block (row 0 has
    // the smallest causal limit, causal_off)
    const int vis_all = p.causal ? min(p.Nk, max(p.causal_off + 1, 0)) : p.Nk;
    float* red = reinterpret_cast<float*>(smem + L::kOffRed);
    float* sums = reinterpret_cast<float*>(smem + L::kOffSum);
    // this thread's P column in the buffer's 64-key block key / 64: row r at
    // r/8 * 1024 + (r%8) * 128, 16-byte chunk (key%64)/8 XOR r%8
    const int kc = t & 63;
    uint8_t* pcol = smem + L::kOffP + (t >> 6) * L::kPRows + (kc & 7) * 2;
    const int chunk = kc >> 3;
    const long long n_rows = static_cast<long long>(p.B) * p.heads * p.Nq;
    // PV of tile c (from P buffer c & 1) has completed
    auto wait_pv = [&](int c, int site) {
      return __all_sync(0xffffffffu,
                        dec_wait(bar(L::kBarPV + (c & 1)), (c >> 1) & 1, wc, site));
    };
    // the item whose epilogue is pending: its head, split, row maxima and sums
    bool pend = false;
    int pend_bh = 0, pend_sp = 0;
    float pend_m[RP], pend_l[RP];
    // Epilogue of an item (all softmax warps; thread t holds column t of O,
    // one TMEM column per query row, its RP rows): O / l to the output (one split) or the split
    // workspace, coalesced along d.  Deferred to the next item's first tile,
    // whose softmax waits for the item's last PV anyway.
    auto epilogue = [&](int bh, int sp) {
      const float(&mq)[RP] = pend_m;
      const float(&lq)[RP] = pend_l;
      ptx::tc_fence_after();
      uint32_t u[16];
      ld_rows(L::tO, u);
      ptx::tmem_wait_ld();
      pin_after_wait<16>(u);
      ptx::tc_fence_before();
#pragma unroll
      for (int q = 0; q < RP; ++q) {
        const int qg = q0 + q;
        if (qg >= nrows) break;
        const float inv_l = (lq[q] > 0.f) ? 1.0f / lq[q] : 0.f;
        const long long row = static_cast<long long>(bh) * p.Nq + qg;
        const float val = __uint_as_float(u[q]) * inv_l;
        const bool lse_thread = t == qg;
        float lse_row = 0.f;
        if (lse_thread) {
          const float m_use = (mq[q] == -INFINITY) ? 0.f : mq[q];
          lse_row = (lq[q] > 0.f) ? (m_use + __log2f(lq[q])) * 0.69314718055994530942f : -INFINITY;
        }
        if (p.n_splits == 1) {
          if (t < D) reinterpret_cast<T*>(p.o)[row * D + t] = T(val);
          if (lse_thread && p.lse != nullptr) p.lse[row] = lse_row;
        } else {
          const size_t ws_row = static_cast<size_t>(sp) * n_rows + row;
          if (t < D) p.ws_o[ws_row * D + t] = val;
          if (lse_thread) p.ws_lse[ws_row] = lse_row;
        }
      }
    };
    // `ok` is this thread's status since the last named barrier; every
    // barrier ANDs it over the softmax warps, so they stop at the same barrier
    // (a thread whose wait failed skips its work but still reaches it).
    bool ok = true;
    int c = 0;
    bool run = true;
    for (int w = blockIdx.x; run && w < n_work; w += gridDim.x) {
      DecItem it;
      dec_item(p, w, it);
      if (it.n == 0) {
        // a lone split without visible keys: O = 0, LSE = -inf
        if (p.n_splits == 1) {
          for (int qg = q0; qg < min(nrows, q0 + RP); ++qg) {
            const long long row = static_cast<long long>(it.bh) * p.Nq + qg;
            if (t < D) reinterpret_cast<T*>(p.o)[row * D + t] = T(0.f);
            if (t == qg && p.lse != nullptr) p.lse[row] = -INFINITY;
          }
        }
        continue;
      }
      float m[RP], l[RP];
#pragma unroll
      for (int q = 0; q < RP; ++q) {
        m[q] = -INFINITY;
        l[q] = 0.f;
      }
      const int nr = (it.n + H - 1) / H;  // rounds of kKeys keys
      for (int j = 0; j < nr; ++j, ++c) {
        const int b = c & 1;
        float x[H][RP];
#pragma unroll
        for (int h = 0; h < H; ++h)
#pragma unroll
          for (int q = 0; q < RP; ++q) x[h][q] = -INFINITY;
        if (ok) ok = __all_sync(0xffffffffu, dec_wait(bar(L::kBarS + b), (c >> 1) & 1, wc, 50));
        if (threadIdx.x == 0) FA_TRACE_AT(c, 4);
        if (ok) {
          ptx::tc_fence_after();
          uint32_t u[H][16];
#pragma unroll
          for (int h = 0; h < H; ++h) ld_rows(L::tS(b) + 16 * h, u[h]);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < H; ++h) pin_after_wait<16>(u[h]);
          ptx::tc_fence_before();
          ptx::mbar_arrive(bar(L::kBarSFree + b));
          // scaled scores; -inf for rows past the block and keys a row does not
          // see (keys past the split's tiles in a round are past Nk or past
          // every row's causal limit).  Tiles below vis_all hold no such key:
          // only rows past the block are masked there.
          const int key0 = (it.jb + j * H) * kBlockN;
          if (key0 + L::kKeys <= vis_all) {
#pragma unroll
            for (int h = 0; h < H; ++h)
#pragma unroll
              for (int q = 0; q < RP; ++q)
                x[h][q] = q0 + q < nrows ? __uint_as_float(u[h][q]) * p.scale_log2 : -INFINITY;
          } else {
#pragma unroll
            for (int h = 0; h < H; ++h) {
              const int key = key0 + 128 * h + t;
#pragma unroll
              for (int q = 0; q < RP; ++q) {
                bool vis = q0 + q < nrows && key < p.Nk;
                if (p.causal) vis = vis && key <= (q0 + q) % p.pos_mod + p.causal_off;
                x[h][q] = vis ? __uint_as_float(u[h][q]) * p.scale_log2 : -INFINITY;
              }
            }
          }
          // tile maxima of the rows over the warp's keys
          float v[RP];
#pragma unroll
          for (int q = 0; q < RP; ++q) v[q] = H == 2 ? fmaxf(x[0][q], x[H - 1][q]) : x[0][q];
          const float wmax = dec_reduce<RP, true>(v, lane);
          if (!(lane & dec_low<RP>())) red[(b * 4 * RS + warp) * RP + dec_row<RP>(lane)] = wmax;
        }
        if (!(ok = ptx::bar_and(L::kNamedBar, kSoftThreads, ok))) {
          run = false;
          break;
        }
        if (threadIdx.x == 0) FA_TRACE_AT(c, 5);
        float mt[RP];
        {
          // the four warps that hold this thread's rows
          const float4* r4 = reinterpret_cast<const float4*>(red + (b * 4 * RS + (warp & ~3)) * RP);
#pragma unroll
          for (int i = 0; i < RP / 4; ++i) {
            const float4 a = r4[i], e = r4[RP / 4 + i], f = r4[2 * (RP / 4) + i], g = r4[3 * (RP / 4) + i];
            mt[4 * i] = fmaxf(fmaxf(a.x, e.x), fmaxf(f.x, g.x));
            mt[4 * i + 1] = fmaxf(fmaxf(a.y, e.y), fmaxf(f.y, g.y));
            mt[4 * i + 2] = fmaxf(fmaxf(a.z, e.z), fmaxf(f.z, g.z));
            mt[4 * i + 3] = fmaxf(fmaxf(a.w, e.w), fmaxf(f.w, g.w));
          }
        }
        // lazy rescale (the same threshold as the attention kernel); every
        // thread holds the same m, so the branches are uniform.  A row's max
        // moves only when it grows past the threshold, which after the first
        // tile is rare: the factors are computed in that branch only.
        bool grow_any = false;
#pragma unroll
        for (int q = 0; q < RP; ++q) grow_any |= mt[q] > m[q] + kRescaleThreshold;
        if (grow_any) {
          float alpha[RP];
#pragma unroll
          for (int q = 0; q < RP; ++q) {
            const bool grow = mt[q] > m[q] + kRescaleThreshold;
            alpha[q] = (grow && j > 0) ? ptx::ex2_approx(m[q] - mt[q]) : 1.0f;
            if (grow) m[q] = mt[q];
          }
          if (j > 0) {
#pragma unroll
            for (int q = 0; q < RP; ++q) l[q] *= alpha[q];
            // O^T holds PV of tiles < j once PV(c-1) completed; PV(c) waits
            // for P(c).  Column q of this thread's lane scales by alpha[q].
            if ((ok = wait_pv(c - 1, 52))) {
              ptx::tc_fence_after();
              uint32_t u[16];
              ld_rows(L::tO, u);
              ptx::tmem_wait_ld();
              pin_after_wait<16>(u);
#pragma unroll
              for (int q = 0; q < RP; ++q) u[q] = __float_as_uint(__uint_as_float(u[q]) * alpha[q]);
              st_rows(L::tO, u);
              ptx::tmem_wait_st();
              ptx::tc_fence_before();
            }
          }
        }
        if (ok && pend) {
          // the previous item's last PV (tile c-1) completed: read its O, then
          // let this item's first PV overwrite the accumulator
          if ((ok = wait_pv(c - 1, 53))) {
            epilogue(pend_bh, pend_sp);
            ptx::mbar_arrive(bar(L::kBarOFree));
          }
          pend = false;
        }
        // P buffer b was last read by PV(c-2)
        if (ok && c >= 2) ok = wait_pv(c - 2, 54);
        if (threadIdx.x == 0) FA_TRACE_AT(c, 7);
        if (ok) {
#pragma unroll
          for (int h = 0; h < H; ++h)
#pragma unroll
            for (int q = 0; q < RP; ++q) {
              const int qg = q0 + q;
              const float e = ptx::ex2_approx(x[h][q] - (m[q] == -INFINITY ? 0.f : m[q]));
              l[q] += e;
              *reinterpret_cast<T*>(pcol + b * L::kPBuf + h * 2 * L::kPRows + (qg >> 3) * 1024 +
                                    (qg & 7) * 128 + ((chunk ^ (qg & 7)) << 4)) = T(e);
            }
          ptx::fence_proxy_async_smem();
          ptx::mbar_arrive(bar(L::kBarP + b));
          if (threadIdx.x == 0) FA_TRACE_AT(c, 6);
        }
      }
      if (!run) break;

      // ---- end of the item: row sums over the 128 keys (the O readout is
      // deferred to the next item's first tile)
      const float wsum = dec_reduce<RP, false>(l, lane);
      if (!(lane & dec_low<RP>())) sums[warp * RP + dec_row<RP>(lane)] = wsum;
      if (!(ok = ptx::bar_and(L::kNamedBar, kSoftThreads, ok))) break;
      // the sums are read before the next item's first barrier, after which
      // they may be overwritten
      {
        const float4* s4 = reinterpret_cast<const float4*>(sums + (warp & ~3) * RP);
#pragma unroll
        for (int i = 0; i < RP / 4; ++i) {
          const float4 a = s4[i], e = s4[RP / 4 + i], f = s4[2 * (RP / 4) + i], g = s4[3 * (RP / 4) + i];
          pend_l[4 * i] = (a.x + e.x) + (f.x + g.x);
          pend_l[4 * i + 1] = (a.y + e.y) + (f.y + g.y);
          pend_l[4 * i + 2] = (a.z + e.z) + (f.z + g.z);
          pend_l[4 * i + 3] = (a.w + e.w) + (f.w + g.w);
        }
#pragma unroll
        for (int q = 0; q < RP; ++q) pend_m[q] = m[q];
      }
      pend_bh = it.bh;
      pend_sp = it.sp;
      pend = true;
    }
    if (ok && pend && wait_pv(c - 1, 53)) epilogue(pend_bh, pend_sp);
  }

  // ---- teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) FA_TRACE_AT(kTraceTiles - 1, 31);
  if (warp == kDecWarpMma) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, L::kTmemCols);
  }
}

template <int D, bool BF16, int R, int RS>
cudaError_t launch_decode_impl(const FwdParams& p, int grid, cudaStream_t stream) {
  auto kern = fa_decode_kernel<D, BF16, R, RS>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               DecLayout<D>::kDynBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  kern<<<grid, 32 * (4 * RS + 2), DecLayout<D>::kDynBytes, stream>>>(p);
  return cudaGetLastError();
}

// the smallest row count (4, 8, 16) that holds the block; 8 rows are split
// between two softmax warpgroups and 16 rows between four, 4 rows per thread
// (measured against one warpgroup holding all rows: 1.08-1.11x for 8 rows;
// 16 rows 1.26-1.46x over two warpgroups, 1.06-1.08x more over four)
template <int D, bool BF16>
cudaError_t launch_decode_rows(const FwdParams& p, int grid, cudaStream_t stream) {
  if (p.Nq <= 4) return launch_decode_impl<D, BF16, 4, 1>(p, grid, stream);
  if (p.Nq <= 8) return launch_decode_impl<D, BF16, 8, 2>(p, grid, stream);
  return launch_decode_impl<D, BF16, 16, 4>(p, grid, stream);
}

}  // namespace

cudaError_t launch_decode(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream) {
  if (p.Nq > kDecRows) return cudaErrorInvalidValue;
  const int n_work = p.B * p.heads * p.n_splits;
  const int grid = (p.n_ctas > 0 && p.n_ctas < n_work) ? p.n_ctas : n_work;
  if (head_dim == 64)
    return bf16 ? launch_decode_rows<64, true>(p, grid, stream)
                : launch_decode_rows<64, false>(p, grid, stream);
  return bf16 ? launch_decode_rows<128, true>(p, grid, stream)
              : launch_decode_rows<128, false>(p, grid, stream);
}

}  // namespace fa
