// Attention forward, "tile" kernel: one 128-row Q tile per work item, with
// the score tile S double-buffered in tensor memory so that the tensor core
// computes S(j+1) while the softmax works on S(j).
//
// Included by fa_fwd_sm100.cu (same translation unit: FwdParams, WorkItem,
// the bounded waits and the softmax helpers are shared with the pair kernel).
//
// Why: in the pair kernel (two Q tiles ping-ponging on one S buffer each) a
// group's chain per K/V tile is PV(j) -> S(j+1) -> softmax(j+1), so the
// softmax waits for two products every tile.  Here S(j+1) goes to the other
// buffer while softmax(j) runs, and PV(j) / S(j+2) run while softmax(j+1)
// runs: the softmax never waits for a product in steady state, and the
// tensor core never waits for more than one softmax.
//
// The softmax of a tile is split between kSplit warpgroups (kSplit = 2 or 4):
// warps w, w + 4, ... read the same TMEM lanes (query rows) and take
// 128 / kSplit consecutive keys each; they exchange row maxima through
// shared memory once per tile.
//   warps 0 .. 4*kSplit-1   softmax (rows = TMEM lanes, key part h = warp / 4)
//   warp  4*kSplit          TMA producer (Q once; K/V ring in the order the MMAs use it)
//   warp  4*kSplit + 1      MMA issuer + TMEM owner
//   2 more warps            idle (complete the warpgroup for setmaxnreg)
//
// Tensor memory (512 columns x 128 lanes, lane = query row):
//   O      [0, d)       fp32 accumulator
//   S_b    [128 + 128b, +128), b = j % 2: S(j) fp32; P(j) (f16/bf16 pairs)
//          overwrites its first 64 columns (part h writes 64/kSplit columns)
//   Q      [384, 384 + d/2)  the Q tile as packed pairs: S = Q K^T reads A
//          from tensor memory and only K from shared memory
//
// Barrier phases: S_b, P_b (parts) and O_b complete once per tile that uses
// buffer b, so a waiter for tile j uses phase j / 2 of buffer j % 2.  Each
// can be at most one phase ahead of any waiter: S(j+2) is issued after PV(j),
// which needs P(j), which needs the softmax to have consumed S(j).

namespace tile {

// -DFA_TRACE timeline of the first kTraceCtas CTAs, events of tile j:
//   0-3  softmax warp 0 (key part 0): S(j) seen, scores loaded and reduced,
//        maxima exchanged, P(j) stored;  4-7 the same for warp 4 (part 1)
//   8    MMA warp: V_j landed;  9 / 10 P(j) parts 0 / last seen;
//   11   K_{j+2} landed;  12 S(j+2) issued
//   13 / 14 producer issued K_j / V_j;  15 producer found K_j's slot free

constexpr int kRows = 128;
constexpr uint32_t kTmemO = 0;
constexpr uint32_t kTmemQ = 384;
__host__ __device__ constexpr uint32_t tmem_s(int b) { return 128u + 128u * static_cast<uint32_t>(b); }

template <int kSplit>
struct TCfg {
  static constexpr int kThreads = 128 * kSplit + 128;
  static constexpr int kWarpLoad = 4 * kSplit;
  static constexpr int kWarpMma = 4 * kSplit + 1;
  static constexpr int kKeys = kBlockN / kSplit;  // keys per thread per tile
  // launch registers (65536 / threads, multiple of 8) and the setmaxnreg split
  // (none with four parts: 96 registers suffice for every role)
  static constexpr int kLaunchRegs = kSplit == 2 ? 168 : 96;
  static constexpr int kRegsSoftmax = kSplit == 2 ? 192 : 96;
  static constexpr int kRegsOther = kSplit == 2 ? 120 : 96;
  static_assert(128 * kSplit * kRegsSoftmax + 128 * kRegsOther <= kThreads * kLaunchRegs,
                "register split exceeds the launch allocation");
};

template <int D, int kSplit>
struct TLayout {
  static constexpr int kColBlocks = D / 64;
  static constexpr int kBlockBytes = kRows * 128;  // one 64-column block of a 128-row tile
  static constexpr int kTile = kRows * D * 2;
  static constexpr int kSlots = (D == 128) ? 5 : 8;
  static constexpr int kOffQ = 0;
  static constexpr int kOffKV = kTile;
  static constexpr int kOffRed = kOffKV + kSlots * kTile;  // float [2 parity][kSplit][128]
  static constexpr int kOffRedL = kOffRed + 2 * kSplit * kRows * 4;  // float [kSplit][128]
  static constexpr int kOffBar = kOffRedL + kSplit * kRows * 4;
  // barrier indices
  static constexpr int kBarQ = 0;                      // Q tile landed (TMA)
  static constexpr int kBarQT = 1;                     // Q copied into TMEM (all softmax threads)
  static constexpr int kBarFull = 2;                   // kSlots
  static constexpr int kBarEmpty = kBarFull + kSlots;  // kSlots
  static constexpr int kBarS = kBarEmpty + kSlots;     // 2 (per S buffer)
  static constexpr int kBarP = kBarS + 2;              // 2 x kSplit (buffer, part): 128 arrivals
  static constexpr int kBarO = kBarP + 2 * kSplit;     // 2 (per buffer of the PV's P)
  static constexpr int kBarDrain = kBarO + 2;
  static constexpr int kNumBars = kBarDrain + 1;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kDynBytes = kBytes + 1024;
  static_assert(kDynBytes <= 227 * 1024, "shared memory budget");
};

// Ring order of a work item with n K/V tiles: the order the MMA warp uses
// them, K0 K1 V0 K2 V1 K3 ... V(n-2) V(n-1) (n = 1: K0 V0).
__device__ __forceinline__ int k_item(int j) { return j < 2 ? j : 2 * j - 1; }
__device__ __forceinline__ int v_item(int j, int n) { return j <= n - 2 ? 2 + 2 * j : 2 * n - 1; }
// inverse: ring item i of the work item -> (is_v, tile)
__device__ __forceinline__ int item_tile(int i, int n, bool& is_v) {
  if (i == 0) { is_v = false; return 0; }
  if (i == 1) { is_v = n == 1; return n == 1 ? 0 : 1; }
  if (i == 2 * n - 1) { is_v = true; return n - 1; }
  is_v = (i & 1) == 0;
  return is_v ? (i - 2) / 2 : (i + 1) / 2;
}

// Work item w of a tile launch: (batch*head, 128-row Q tile, key split).
// p.n_qpairs counts 128-row tiles per (batch, head) here.
__device__ __forceinline__ void decode(const FwdParams& p, int w, WorkItem& it) {
  it.sp = w % p.n_splits;
  int qt;
  item_order(p, w / p.n_splits, qt, it.bh);
  if (p.causal) qt = p.n_qpairs - 1 - qt;  // causal: heaviest tiles first
  it.qp = qt;
  const int b = it.bh / p.heads;
  const int hq = it.bh % p.heads;
  it.bh_kv = b * p.Hkv + hq / p.group;
  it.q_row0 = qt * kRows;
  int n_kv_tiles = p.n_kv_tiles;
  if (p.ranges == 0) {
    it.nq = p.Nq;
    it.nk = p.Nk;
    it.causal_off = p.causal_off;
    it.qy = 0;
    it.qz = it.bh;
    it.ky = 0;
    it.kz = it.bh_kv;
  } else {
    const int ql = min(max(__ldg(p.q_lo + b), 0), p.q_lim);
    const int kl = min(max(__ldg(p.k_lo + b), 0), p.k_lim);
    it.nq = min(max(__ldg(p.q_hi + b), ql), p.q_lim) - ql;
    it.nk = min(max(__ldg(p.k_hi + b), kl), p.k_lim) - kl;
    it.ky = kl;
    it.qy = ql;
    if (p.ranges == 1) {
      it.causal_off = p.causal_off + (p.causal_br ? it.nk - it.nq : 0);
      it.qz = hq;
      it.kz = hq / p.group;
    } else {
      it.causal_off = p.causal_off + ql - kl;
      it.qz = it.bh;
      it.kz = it.bh_kv;
    }
    n_kv_tiles = (it.nk + kBlockN - 1) / kBlockN;
  }
  it.has_q1 = false;
  const int total = kv_tiles_core(p.causal, it.nq, n_kv_tiles, it.causal_off, p.pos_mod, qt);
  const int j_begin = it.sp * p.tiles_per_split;
  it.n_kv[0] = max(0, min(total, j_begin + p.tiles_per_split) - j_begin);
  it.n_kv[1] = 0;
  it.jb[0] = it.jb[1] = j_begin;
  it.n_loop = it.n_kv[0];
  it.n_items = 2 * it.n_kv[0];
}

// TMEM <-> registers in chunks of N 32-bit columns (N = 8, 16 or 32)
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 32) ptx::tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  else if constexpr (N == 16) ptx::tmem_ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(r));
  else ptx::tmem_ld8(taddr, r);
}
template <int N>
__device__ __forceinline__ void tmem_st_n(uint32_t taddr, const uint32_t* r) {
  if constexpr (N == 32) ptx::tmem_st32(taddr, *reinterpret_cast<const uint32_t(*)[32]>(r));
  else if constexpr (N == 16) ptx::tmem_st16(taddr, r);
  else ptx::tmem_st8(taddr, r);
}

template <int D, bool BF16, int kSplit>
__global__ void __launch_bounds__(TCfg<kSplit>::kThreads, 1)
    fa_fwd_tile_kernel(const __grid_constant__ FwdParams p) {
  using L = TLayout<D, kSplit>;
  using C = TCfg<kSplit>;
  constexpr int kKeys = C::kKeys;          // keys per thread per tile
  constexpr int kPCols = kKeys / 2;        // packed P columns per thread
  constexpr int kOCols = D / kSplit;       // O columns per thread (rescale, epilogue)
  constexpr int kOChunk = kOCols < 32 ? kOCols : 32;
  constexpr int kQChunks = D / 8 / kSplit;  // 16-byte chunks of a Q row per thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };

  WorkItem it;
  const int w_item = p.item0 + static_cast<int>(blockIdx.x);
  decode(p, w_item, it);
  const int n = it.n_loop;

  if (threadIdx.x == 0) {
    const unsigned long long st = *reinterpret_cast<volatile unsigned long long*>(&g_fa_status);
    *abort_flag = ((st >> 32) == p.epoch && (st & 0xffffffffull) != 0ull) ? 1 : 0;
    for (int i = 0; i < L::kNumBars; ++i) {
      uint32_t count = 1;
      if (i == L::kBarQT) count = 128 * kSplit;
      if (i >= L::kBarP && i < L::kBarP + 2 * kSplit) count = 128;
      ptx::mbar_init(bar(i), count);
    }
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (*abort_flag) return;
  if (warp == C::kWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), 512);
    ptx::tmem_relinquish();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};
  if (threadIdx.x == 0) FA_TRACE_AT(kTraceTiles - 1, 30);  // CTA set up

  if (warp >= 4 * kSplit) {
    // -------------------------------------------------- producer warpgroup
    if constexpr (C::kRegsOther != C::kLaunchRegs) ptx::setmaxnreg_dec<C::kRegsOther>();
    if (warp == C::kWarpLoad && lane == 0 && n > 0) {
      ptx::prefetch_tmap(&p.tm_q);
      ptx::prefetch_tmap(&p.tm_k);
      ptx::prefetch_tmap(&p.tm_v);
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_last();
      const bool skip_q = (p.debug_flags & FA_DEBUG_SKIP_Q_LOAD) != 0;
      if (!skip_q) {
        ptx::mbar_arrive_expect_tx(bar(L::kBarQ), L::kTile);
        const int row = it.qy + it.q_row0;
#pragma unroll
        for (int c = 0; c < L::kColBlocks; ++c) {
          if (p.ranges == 1)
            ptx::tma_load_3d(sbase + L::kOffQ + c * L::kBlockBytes, &p.tm_q, bar(L::kBarQ), c * 64,
                             it.qz, row, pol_q);
          else
            ptx::tma_load_3d(sbase + L::kOffQ + c * L::kBlockBytes, &p.tm_q, bar(L::kBarQ), c * 64,
                             row, it.qz, pol_q);
        }
      }
      int i = 0;
      for (; i < 2 * n; ++i) {
        const int slot = i % L::kSlots;
        bool is_v;
        const int jt = item_tile(i, n, is_v);
        if (i >= L::kSlots && !bar_wait(bar(L::kBarEmpty + slot), ((i / L::kSlots) - 1) & 1, wc, 1))
          break;
        if (!is_v) FA_TRACE_AT(jt, 15);
        const int tile = it.jb[0] + jt;
        const uint32_t dst = sbase + L::kOffKV + slot * L::kTile;
        const void* map = is_v ? static_cast<const void*>(&p.tm_v) : static_cast<const void*>(&p.tm_k);
        ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile);
        const int row = it.ky + tile * kBlockN;
#pragma unroll
        for (int c = 0; c < L::kColBlocks; ++c) {
          if (p.ranges == 1)
            ptx::tma_load_3d(dst + c * L::kBlockBytes, map, bar(L::kBarFull + slot), c * 64, it.kz,
                             row, pol_kv);
          else
            ptx::tma_load_3d(dst + c * L::kBlockBytes, map, bar(L::kBarFull + slot), c * 64, row,
                             it.kz, pol_kv);
        }
        FA_TRACE_AT(jt, is_v ? 14 : 13);
      }
      // every copy this thread started lands before the CTA exits
      for (int r = max(0, i - L::kSlots); r < i; ++r)
        bar_wait(bar(L::kBarFull + r % L::kSlots), (r / L::kSlots) & 1, wc, 2, false);
      if (!skip_q) bar_wait(bar(L::kBarQ), 0, wc, 2, false);
    } else if (warp == C::kWarpMma && n > 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t fmt = BF16 ? 1u : 0u;
      constexpr uint32_t idesc_qk = ptx::make_idesc_f16(kRows, kBlockN, fmt, 0, 0);
      constexpr uint32_t idesc_pv = ptx::make_idesc_f16(kRows, D, fmt, 0, 1);
      constexpr int kSteps = 8 / kSplit;  // PV K-steps (16 keys) per softmax part
      auto slot_of = [](int item) { return item % L::kSlots; };
      auto phase_of = [](int item) { return static_cast<uint32_t>((item / L::kSlots) & 1); };
      const uint64_t k_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, 16, 1024);
      const uint64_t v_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, L::kBlockBytes, 1024);
      auto wait = [&](uint32_t b, uint32_t ph, int site) {
        return __all_sync(0xffffffffu, bar_wait(b, ph, wc, site));
      };
      auto commit = [&](uint32_t b) {
        if (ptx::elect_one()) ptx::mma_commit(b);
        __syncwarp();
      };
      // S(j) = Q K_j^T into buffer j % 2 (A = Q from TMEM, B = K K-major)
      auto issue_s = [&](int j) -> bool {
        const int ki = k_item(j);
        if (!wait(bar(L::kBarFull + slot_of(ki)), phase_of(ki), 11)) return false;
        if (lane == 0 && j >= 2) FA_TRACE_AT(j - 2, 11);
        ptx::tc_fence_after();
        const uint64_t kd = k_desc0 + static_cast<uint64_t>((slot_of(ki) * L::kTile) >> 4);
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
            ptx::mma_ts(tmem + tmem_s(j & 1), tmem + kTmemQ + 8 * kk, kd + off, idesc_qk,
                        kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(bar(L::kBarS + (j & 1)));
          ptx::mma_commit(bar(L::kBarEmpty + slot_of(ki)));
        }
        __syncwarp();
        if (lane == 0 && j >= 2) FA_TRACE_AT(j - 2, 12);
        return true;
      };
      bool ok = wait(bar(L::kBarQT), 0, 10);
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int j = 0; ok && j < n; ++j) {
        const int b = j & 1;
        const uint32_t ph = static_cast<uint32_t>((j >> 1) & 1);
        const int vi = v_item(j, n);
        if (!(ok = wait(bar(L::kBarFull + slot_of(vi)), phase_of(vi), 12))) break;
        if (lane == 0) FA_TRACE_AT(j, 8);
        const uint64_t vd = v_desc0 + static_cast<uint64_t>((slot_of(vi) * L::kTile) >> 4);
        // O += P(j) V_j, each part's keys once that part has stored its P
#pragma unroll
        for (int h = 0; h < kSplit; ++h) {
          if (!(ok = wait(bar(L::kBarP + kSplit * b + h), ph, 13 + (h & 1)))) break;
          if (lane == 0 && (h == 0 || h == kSplit - 1)) FA_TRACE_AT(j, h == 0 ? 9 : 10);
          ptx::tc_fence_after();
          if (ptx::elect_one()) {
#pragma unroll
            for (int kk = kSteps * h; kk < kSteps * h + kSteps; ++kk)
              ptx::mma_ts(tmem + kTmemO, tmem + tmem_s(b) + kk * 8,
                          vd + static_cast<uint64_t>((kk * 2048) >> 4), idesc_pv,
                          (j > 0 || kk > 0) ? 1u : 0u);
          }
          __syncwarp();
        }
        if (!ok) break;
        commit(bar(L::kBarO + b));
        commit(bar(L::kBarEmpty + slot_of(vi)));
        if (j + 2 < n) ok = issue_s(j + 2);
      }
      commit(bar(L::kBarDrain));
      bar_wait(bar(L::kBarDrain), 0, wc, 19, false);
      __syncwarp();
    }
  } else {
    // -------------------------------------------------- softmax warps
    if constexpr (C::kRegsSoftmax != C::kLaunchRegs) ptx::setmaxnreg_inc<C::kRegsSoftmax>();
    const int h = warp >> 2;                 // key part of every tile
    const int wq = warp & 3;
    const int r = wq * 32 + lane;            // row of the Q tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t named = 1u + static_cast<uint32_t>(wq);  // warps wq, wq + 4, ...
    constexpr uint32_t kNamedCount = 32 * kSplit;
    float* red = reinterpret_cast<float*>(smem + L::kOffRed);
    float* red_l = reinterpret_cast<float*>(smem + L::kOffRedL);
    const float sl = p.scale_log2;
    const int q_row = it.q_row0 + r;
    bool ok = true;

    // Q tile (128-byte swizzle: 16-byte chunk c of row r at c ^ (r % 8)) into
    // TMEM lane r as packed pairs; part h copies chunks [h*kQChunks, +kQChunks)
    if (n > 0) {
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarQ), 0, wc, 9));
      if (ok) {
        uint32_t w[4 * kQChunks];
#pragma unroll
        for (int c = 0; c < kQChunks; ++c) {
          const int cg = h * kQChunks + c;  // chunk of the row (8 per 64-column block)
          const uint4 v = *reinterpret_cast<const uint4*>(
              smem + L::kOffQ + (cg >> 3) * L::kBlockBytes + r * 128 + (((cg & 7) ^ (r & 7)) * 16));
          w[4 * c] = v.x;
          w[4 * c + 1] = v.y;
          w[4 * c + 2] = v.z;
          w[4 * c + 3] = v.w;
        }
        tmem_st_n<4 * kQChunks>(tmem + lane_off + kTmemQ + 4 * kQChunks * h, w);
        ptx::tmem_wait_st();
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarQT));
    }

    // keys visible to this row: k < row_end; tile_end: the smallest limit over
    // the tile's rows (a key part needs masking when any key reaches it)
    int row_end = it.nk;
    int tile_end = it.nk;
    if (p.causal) {
      row_end = min(row_end, q_row % p.pos_mod + it.causal_off + 1);
      const int lo = it.q_row0;
      const int hi = min(lo + kRows - 1, it.nq - 1);
      const int min_pos = (p.pos_mod >= it.nq) ? lo
                          : (hi / p.pos_mod != lo / p.pos_mod) ? 0
                                                                : lo % p.pos_mod;
      tile_end = min(tile_end, min_pos + it.causal_off + 1);
    }

    float m = -INFINITY;  // running row max (log2 units), the same in every part
    float l = 0.f;        // this part's running sum of exp2(s - m)
    for (int j = 0; j < n; ++j) {
      const int b = j & 1;
      if (ok) ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + b), (j >> 1) & 1, wc, 20 + (h & 1)));
      const bool tr = (wq == 0 && lane == 0 && h < 2);
      if (tr) FA_TRACE_AT(j, 4 * h + 0);
      float x[kKeys];
      float pm = -INFINITY;
      const int key0 = (it.jb[0] + j) * kBlockN + kKeys * h;
      const bool masked = key0 + kKeys > tile_end;
      float sl_eff = sl;
      if (ok) {
        ptx::tc_fence_after();
        uint32_t u[kKeys];
#pragma unroll
        for (int c = 0; c < kKeys; c += 32)
          ptx::tmem_ld32(tmem + lane_off + tmem_s(b) + kKeys * h + c,
                         *reinterpret_cast<uint32_t(*)[32]>(u + c));
        ptx::tmem_wait_ld();
        pin_after_wait<kKeys>(u);
#pragma unroll
        for (int c = 0; c < kKeys; ++c) x[c] = __uint_as_float(u[c]);
        // partial maximum of this part in scaled (log2) units
        if (masked) {
          const int lim = row_end - key0;
#pragma unroll
          for (int c = 0; c < kKeys; c += 2) ptx::fmul2(x[c], x[c + 1], x[c], x[c + 1], sl, sl);
#pragma unroll
          for (int c = 0; c < kKeys; ++c)
            if (c >= lim) x[c] = -INFINITY;
          pm = row_extreme<kKeys, false>(x);
          sl_eff = 1.0f;
        } else if (sl >= 0.f) {
          pm = row_extreme<kKeys, false>(x) * sl;
        } else {
          pm = row_extreme<kKeys, true>(x) * sl;
        }
        red[(b * kSplit + h) * kRows + r] = pm;
        if (tr) FA_TRACE_AT(j, 4 * h + 1);
      }
      // Every part of a row has read its scores (so P may overwrite them) and
      // published its maximum.  A failed wait in any of the warps makes all of
      // them leave here, at the same barrier.
      if (!ptx::bar_and(named, kNamedCount, ok)) {
        ok = false;
        break;
      }
      if (tr) FA_TRACE_AT(j, 4 * h + 2);
      float m_tile = pm;
#pragma unroll
      for (int o = 0; o < kSplit; ++o)
        if (o != h) m_tile = fmaxf(m_tile, red[(b * kSplit + o) * kRows + r]);
      const float m_new = fmaxf(m, m_tile);
      const bool grow = m_new > m + kRescaleThreshold;
      if (j == 0) {
        m = m_new;
      } else if (__any_sync(0xffffffffu, grow)) {
        // O holds PV(0..j-1) once PV(j-1) has completed; this part rescales
        // its d/kSplit columns.  The warps of a row quad hold the same rows
        // and maxima, so all take this branch, and the barrier below keeps
        // PV(j) -- which writes all d columns and may start on part 0's P
        // alone -- behind every part's rescale.
        ok = __all_sync(0xffffffffu,
                        bar_wait(bar(L::kBarO + ((j - 1) & 1)), ((j - 1) >> 1) & 1, wc, 24 + (h & 1)));
        const float alpha = grow ? ptx::ex2_approx(m - m_new) : 1.0f;
        if (ok) {
          ptx::tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kOCols; c += kOChunk) {
            uint32_t o[kOChunk];
            const uint32_t col = kTmemO + kOCols * h + c;
            tmem_ld_n<kOChunk>(tmem + lane_off + col, o);
            ptx::tmem_wait_ld();
            pin_after_wait<kOChunk>(o);
#pragma unroll
            for (int i = 0; i < kOChunk; i += 2) {
              float a0 = __uint_as_float(o[i]), a1 = __uint_as_float(o[i + 1]);
              ptx::fmul2(a0, a1, a0, a1, alpha, alpha);
              o[i] = __float_as_uint(a0);
              o[i + 1] = __float_as_uint(a1);
            }
            tmem_st_n<kOChunk>(tmem + lane_off + col, o);
          }
          ptx::tmem_wait_st();
        }
        ptx::tc_fence_before();
        if (ptx::bar_and(named, kNamedCount, ok)) {
          ptx::tc_fence_after();
          if (grow) {
            l *= alpha;
            m = m_new;
          }
        } else {
          ok = false;
        }
      }
      if (!ok) continue;  // leaves at the next barrier (or the final one)
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      // P = exp2(x * sl_eff - m) as packed pairs over this part's columns
      float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
      for (int q = 0; q < kKeys / 32; ++q) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int i = 32 * q + 2 * c;
          float e0, e1;
          if (masked)
            exp2_pair<false>(c, x[i], x[i + 1], sl_eff, neg_m, e0, e1);
          else
            exp2_pair<true>(c, x[i], x[i + 1], sl_eff, neg_m, e0, e1);
          if (c & 1)
            ptx::fadd2(b0, b1, b0, b1, e0, e1);
          else
            ptx::fadd2(a0, a1, a0, a1, e0, e1);
          pk[c] = pack2<BF16>(e0, e1);
        }
        ptx::tmem_st16(tmem + lane_off + tmem_s(b) + kPCols * h + 16 * q, pk);
      }
      ptx::fadd2(a0, a1, a0, a1, b0, b1);
      l += a0 + a1;
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarP + kSplit * b + h));
      if (tr) FA_TRACE_AT(j, 4 * h + 3);
    }

    // ---- epilogue: row sum over all parts, O / l, LSE
    red_l[h * kRows + r] = l;
    const bool all_ok = ptx::bar_and(named, kNamedCount, ok);
    ok = ok && all_ok;
    float l_tot = 0.f;
#pragma unroll
    for (int o = 0; o < kSplit; ++o) l_tot += red_l[o * kRows + r];
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    long long o_row0, lse_row0;
    int nq;
    item_out(p, w_item, o_row0, lse_row0, nq);
    const bool row_ok = q_row < nq;
    const size_t row_index = static_cast<size_t>(lse_row0) + q_row;
    T* const orow = reinterpret_cast<T*>(p.o) + o_row0 + static_cast<long long>(q_row) * p.o_rs;
    const long long lse_index = lse_row0 + q_row;
    const bool partial = p.n_splits > 1;
    if (n == 0) {
      // no visible key: O = 0, LSE = -inf (a split without tiles leaves its
      // rows to the other splits)
      if (!partial && row_ok) {
        uint4* dst = reinterpret_cast<uint4*>(orow + kOCols * h);
#pragma unroll
        for (int i = 0; i < kOCols / 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
        if (h == 0 && p.lse != nullptr) p.lse[lse_index] = -INFINITY;
      }
    } else if (ok) {
      ok = __all_sync(0xffffffffu,
                      bar_wait(bar(L::kBarO + ((n - 1) & 1)), ((n - 1) >> 1) & 1, wc, 22 + (h & 1)));
      if (ok) {
        ptx::tc_fence_after();
        const float inv_l = (l_tot > 0.f) ? 1.0f / l_tot : 0.f;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        const float lse_row =
            (l_tot > 0.f) ? (m_use + __log2f(l_tot)) * 0.69314718055994530942f : -INFINITY;
        if (!partial) {
#pragma unroll
          for (int c = 0; c < kOCols; c += kOChunk) {
            uint32_t o[kOChunk];
            tmem_ld_n<kOChunk>(tmem + lane_off + kTmemO + kOCols * h + c, o);
            ptx::tmem_wait_ld();
            pin_after_wait<kOChunk>(o);
            uint32_t hv[kOChunk / 2];
#pragma unroll
            for (int i = 0; i < kOChunk / 2; ++i)
              hv[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l,
                                  __uint_as_float(o[2 * i + 1]) * inv_l);
            if (row_ok) {
              uint4* dst = reinterpret_cast<uint4*>(orow + kOCols * h + c);
#pragma unroll
              for (int i = 0; i < kOChunk / 8; ++i)
                dst[i] = make_uint4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
            }
          }
          if (h == 0 && row_ok && p.lse != nullptr) p.lse[lse_index] = lse_row;
        } else {
          // partial result of this key split, normalised by its own row sum
          const size_t ws_row = static_cast<size_t>(it.sp) * p.B * p.heads * p.Nq + row_index;
          float* wrow = p.ws_o + ws_row * D + kOCols * h;
#pragma unroll
          for (int c = 0; c < kOCols; c += kOChunk) {
            uint32_t o[kOChunk];
            tmem_ld_n<kOChunk>(tmem + lane_off + kTmemO + kOCols * h + c, o);
            ptx::tmem_wait_ld();
            pin_after_wait<kOChunk>(o);
            if (row_ok) {
              float4* dst = reinterpret_cast<float4*>(wrow + c);
#pragma unroll
              for (int i = 0; i < kOChunk / 4; ++i)
                dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l,
                                     __uint_as_float(o[4 * i + 1]) * inv_l,
                                     __uint_as_float(o[4 * i + 2]) * inv_l,
                                     __uint_as_float(o[4 * i + 3]) * inv_l);
            }
          }
          if (h == 0 && row_ok) p.ws_lse[ws_row] = lse_row;
        }
      }
    }
  }

  // ---- teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) FA_TRACE_AT(kTraceTiles - 1, 31);  // CTA done
  if (warp == C::kWarpMma) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace tile
