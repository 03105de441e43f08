// Attention forward at d = 128 on CTA pairs: the pair kernel's schedule (two
// 128-row Q tiles per CTA, softmax groups ping-ponging on the tensor pipe)
// with every product issued once for two SMs (tcgen05 cta_group::2, M = 256).
//
// Included by fa_fwd_sm100.cu (shares FwdParams, WorkItem, the bounded waits,
// the softmax helpers and exp_tile's arithmetic with the one-SM kernels).
//
// A cluster of two CTAs owns a "Q quad": 512 consecutive query rows of one
// (batch, head).  CTA r holds Q tiles 4q + r (group 0) and 4q + 2 + r
// (group 1), so group g's product covers the 256 contiguous rows
// 512q + 256g .. +255, CTA 0's 128 of them first.  Per K/V tile:
//   S_g  = Q_g K^T   M = 256 (each CTA's Q tile from its own shared memory),
//                    N = 128 keys: each CTA holds 64 of them (K rows 64r..)
//   O_g += P_g V     A = P_g from each CTA's tensor memory, N = d = 128:
//                    each CTA holds V's columns 64r .. 64r + 63
// so each SM streams half of every K and V tile and the pair issues half the
// product instructions of two one-SM CTAs; the shared-memory reads of a
// score product drop from 8 KB to 6 KB per SM.
//
// Roles (both CTAs, 384 threads): warps 0-7 softmax groups, warp 8 TMA
// producer, warp 9 the MMA issuer in CTA 0 (idle in CTA 1) and TMEM owner.
// CTA 0's barriers gate the products: both producers' loads count their
// bytes on CTA 0's "full" barriers, and CTA 1's softmax threads arrive on
// CTA 0's P barriers.  CTA 0's commits arrive on the S, O and ring "empty"
// barriers of both CTAs.  Every wait is bounded; both CTAs meet once more,
// through an mbarrier handshake with a bounded wait, before freeing the
// pair's tensor memory.

namespace pair2 {

constexpr int D = 128;
constexpr uint16_t kBoth = 0x3;  // both CTAs of the pair

struct PLayout {
  static constexpr int kBlockBytes = kBlockM * 128;  // 128 rows x 64 columns (Q)
  static constexpr int kTile = kBlockM * D * 2;      // a 128-row Q tile
  static constexpr int kHalf = 16384;  // K: 64 keys x 128 d; V: 128 keys x 64 d columns
  static constexpr int kKBlock = 64 * 128;  // 64 rows x 64 columns of a K half
  static constexpr int kSlots = 9;
  static constexpr int kOffQ = 0;                  // Q tiles of groups 0, 1
  static constexpr int kOffKV = 2 * kTile;         // ring slot s at kOffKV + s*kHalf
  static constexpr int kOffBar = kOffKV + kSlots * kHalf;
  static constexpr int kBarQ = 0;                       // 2 (CTA 0: both CTAs' Q tile g)
  static constexpr int kBarFull = 2;                    // kSlots (CTA 0: both halves)
  static constexpr int kBarEmpty = kBarFull + kSlots;   // kSlots (both CTAs)
  static constexpr int kBarS = kBarEmpty + kSlots;      // 2
  static constexpr int kBarP = kBarS + 2;               // 2 (CTA 0: 256 arrivals)
  static constexpr int kBarO = kBarP + 2;               // 2
  static constexpr int kBarPH = kBarO + 2;              // 2 (CTA 0: 256 arrivals)
  static constexpr int kBarDrain = kBarPH + 2;          // 1
  static constexpr int kBarExit = kBarDrain + 1;        // 1 (the other CTA is done)
  static constexpr int kNumBars = kBarExit + 1;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kDynBytes = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  __host__ __device__ static constexpr uint32_t tS(int g) { return g ? 128u : 0u; }
  __host__ __device__ static constexpr uint32_t tO(int g) { return g ? 384u : 256u; }
  __host__ __device__ static constexpr uint32_t tP(int g) { return tS(g); }  // P overwrites S
  static_assert(kDynBytes <= 227 * 1024, "shared memory budget");
};

// Bounded wait with cluster-scope acquire (phases the other CTA completes).
// `respect_abort` = false waits out an abort too (teardown handshake).
__device__ __forceinline__ bool bar_wait_cluster(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                                 int site, bool respect_abort = true) {
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63u) == 63u) {
      if (respect_abort && *c.abort) return false;
      if (ptx::global_timer_ns() - t0 > c.timeout_ns) {
        *c.abort = 1;
        record_error(c.epoch, FA_ERR_TIMEOUT_BASE + site);
        return false;
      }
    }
  }
}

// Work item of cluster c: (batch*head, Q quad); p.n_qpairs counts quads.
struct Quad {
  int bh, bh_kv, quad;
  int n_kv[2];  // K/V tiles of group g (both CTAs' tiles of the group)
};

__device__ __forceinline__ Quad decode_quad(const FwdParams& p, int c) {
  Quad q;
  int qd;
  item_order(p, c, qd, q.bh);
  if (p.causal) qd = p.n_qpairs - 1 - qd;  // causal: heaviest quads first
  q.quad = qd;
  const int b = q.bh / p.heads;
  q.bh_kv = b * p.Hkv + (q.bh % p.heads) / p.group;
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int t0 = 4 * qd + 2 * g;
    q.n_kv[g] = max(kv_tiles_core(p.causal, p.Nq, p.n_kv_tiles, p.causal_off, p.pos_mod, t0),
                    kv_tiles_core(p.causal, p.Nq, p.n_kv_tiles, p.causal_off, p.pos_mod, t0 + 1));
  }
  return q;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1) fa_fwd_pair2_kernel(const __grid_constant__ FwdParams p) {
  using L = PLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };
  // the same barrier in CTA 0 (where the products are gated)
  auto lead_bar = [&](int i) -> uint32_t { return ptx::mapa(bar(i), 0); };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < L::kNumBars; ++i) {
      const bool two_ctas = (i == L::kBarP || i == L::kBarP + 1 || i == L::kBarPH || i == L::kBarPH + 1);
      ptx::mbar_init(bar(i), two_ctas ? 256u : 1u);
    }
    ptx::fence_barrier_init();
  }
  __syncthreads();
  ptx::cluster_sync();  // both CTAs' barriers exist before either touches the other's
  if (warp == kWarpMma) {
    ptx::tmem_alloc_pair(ptx::smem_u32(tmem_slot), L::kTmemCols);
    ptx::tmem_relinquish_pair();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};

  if (warp >= 8) {
    ptx::setmaxnreg_dec<kRegsOther>();
    const Quad qi = decode_quad(p, p.item0 + static_cast<int>(blockIdx.x >> 1));
    const int n_loop = max(qi.n_kv[0], qi.n_kv[1]);
    if (warp == kWarpLoad && lane == 0 && n_loop > 0) {
      // ================================================= TMA producer
      ptx::prefetch_tmap(&p.tm_q);
      ptx::prefetch_tmap(&p.tm_k);
      ptx::prefetch_tmap(&p.tm_v);
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_last();
      const bool skip_q = (p.debug_flags & FA_DEBUG_SKIP_Q_LOAD) != 0;
      int q_loads[2] = {0, 0};
      for (int g = 0; g < 2 && !skip_q; ++g) {
        if (qi.n_kv[g] == 0) continue;
        if (leader) ptx::mbar_arrive_expect_tx(bar(L::kBarQ + g), 2 * L::kTile);
        const int row = (4 * qi.quad + 2 * g + static_cast<int>(rank)) * kBlockM;
#pragma unroll
        for (int c = 0; c < 2; ++c)
          ptx::tma_load_3d_pair(sbase + L::kOffQ + g * L::kTile + c * L::kBlockBytes, &p.tm_q,
                                lead_bar(L::kBarQ + g), c * 64, row, qi.bh, pol_q);
        ++q_loads[g];
      }
      // ring items K0 V0 K1 V1 ...: this CTA's half of each tile
      const int n_items = 2 * n_loop;
      int i = 0;
      for (; i < n_items; ++i) {
        const int slot = i % L::kSlots;
        if (i >= L::kSlots && !bar_wait(bar(L::kBarEmpty + slot), ((i / L::kSlots) - 1) & 1, wc, 1))
          break;
        if (leader) ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), 2 * L::kHalf);
        const uint32_t dst = sbase + L::kOffKV + slot * L::kHalf;
        const uint32_t full = lead_bar(L::kBarFull + slot);
        const int tile = i >> 1;
        if ((i & 1) == 0) {
          // K rows 128*tile + 64*rank .. +63, all 128 columns (two 64-column blocks)
          const int row = tile * kBlockN + 64 * static_cast<int>(rank);
#pragma unroll
          for (int c = 0; c < 2; ++c)
            ptx::tma_load_3d_pair(dst + c * L::kKBlock, &p.tm_k, full, c * 64, row, qi.bh_kv, pol_kv);
        } else {
          // V rows 128*tile .. +127, columns 64*rank .. +63
          ptx::tma_load_3d_pair(dst, &p.tm_v, full, 64 * static_cast<int>(rank), tile * kBlockN,
                                qi.bh_kv, pol_kv);
        }
      }
      if (leader) {
        // both CTAs' copies land before CTA 0 signals that it is done (their
        // bytes complete these phases)
        for (int r = max(0, i - L::kSlots); r < i; ++r)
          bar_wait(bar(L::kBarFull + r % L::kSlots), (r / L::kSlots) & 1, wc, 2, false);
        for (int g = 0; g < 2; ++g)
          if (q_loads[g] > 0) bar_wait(bar(L::kBarQ + g), 0, wc, 2, false);
      }
    } else if (warp == kWarpMma && leader && n_loop > 0) {
      // ================================================= MMA issuer (CTA 0)
      constexpr uint32_t fmt = BF16 ? 1u : 0u;
      constexpr uint32_t idesc_qk = ptx::make_idesc_f16(2 * kBlockM, kBlockN, fmt, 0, 0);
      constexpr uint32_t idesc_pv = ptx::make_idesc_f16(2 * kBlockM, D, fmt, 0, 1);
      auto slot_of = [](int item) { return item % L::kSlots; };
      auto phase_of = [](int item) { return static_cast<uint32_t>((item / L::kSlots) & 1); };
      const uint64_t k_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, 16, 1024);
      const uint64_t v_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, L::kBlockBytes, 1024);
      const uint64_t q_desc0 = ptx::smem_desc_sw128(sbase + L::kOffQ, 16, 1024);
      const uint64_t q_desc1 = ptx::smem_desc_sw128(sbase + L::kOffQ + L::kTile, 16, 1024);
      auto wait = [&](uint32_t b, uint32_t ph, int site) {
        return __all_sync(0xffffffffu, bar_wait_lean(b, ph, wc, site));
      };
      auto wait_c = wait;
      auto commit = [&](uint32_t b) {
        if (ptx::elect_one()) ptx::mma_commit_pair(b, kBoth);
        __syncwarp();
      };
      // S_g = Q_g K^T: Q blocks are 16 KB apart (128 rows), K-half blocks 8 KB (64 rows)
      auto issue_s = [&](int g, int ki, uint64_t qd) {
        const uint64_t kd = k_desc0 + static_cast<uint64_t>((slot_of(ki) * L::kHalf) >> 4);
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t qo = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
            const uint64_t ko = static_cast<uint64_t>(((kk / 4) * L::kKBlock + (kk % 4) * 32) >> 4);
            ptx::mma_ss_pair(tmem + L::tS(g), qd + qo, kd + ko, idesc_qk, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit_pair(bar(L::kBarS + g), kBoth);
        }
        __syncwarp();
      };
      // O_g (+)= P_g V: the early quarters of P (both CTAs announced them on
      // PH), then the rest after P
      auto issue_pv = [&](int g, int vi, bool first, uint32_t ph) -> bool {
        const uint64_t vd = v_desc0 + static_cast<uint64_t>((slot_of(vi) * L::kHalf) >> 4);
        if (!wait_c(bar(L::kBarPH + g), ph, 13 + 3 * g)) return false;
        ptx::tc_fence_after();
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 2 * kPEarlyQuarters; ++kk)
            ptx::mma_ts_pair(tmem + L::tO(g), tmem + L::tP(g) + kk * 8,
                             vd + static_cast<uint64_t>((kk * 2048) >> 4), idesc_pv,
                             (!first || kk > 0) ? 1u : 0u);
        }
        __syncwarp();
        if (!wait_c(bar(L::kBarP + g), ph, 13 + 3 * g)) return false;
        ptx::tc_fence_after();
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 2 * kPEarlyQuarters; kk < kBlockN / 16; ++kk)
            ptx::mma_ts_pair(tmem + L::tO(g), tmem + L::tP(g) + kk * 8,
                             vd + static_cast<uint64_t>((kk * 2048) >> 4), idesc_pv, 1u);
          ptx::mma_commit_pair(bar(L::kBarO + g), kBoth);
        }
        __syncwarp();
        return true;
      };
      // Issue order per tile j (as the one-SM pair kernel):
      //   PV0(j)  S0(j+1)  PV1(j)  S1(j+1)
      // S_g(j+1) overwrites P_g(j) after PV_g(j) has read it (in-order products).
      const bool g0 = qi.n_kv[0] > 0;
      const bool g1 = qi.n_kv[1] > 0;
      bool ok = true;
      if (g0) ok = wait(bar(L::kBarQ), 0, 10);
      if (ok && g1) ok = wait(bar(L::kBarQ + 1), 0, 10);
      if (ok) ok = wait(bar(L::kBarFull + slot_of(0)), phase_of(0), 11);
      if (ok) {
        ptx::tc_fence_after();
        if (g0) issue_s(0, 0, q_desc0);
        if (g1) issue_s(1, 0, q_desc1);
        commit(bar(L::kBarEmpty + slot_of(0)));
      }
      for (int j = 0; ok && j < n_loop; ++j) {
        const int item_v = 2 * j + 1;
        const int item_k = 2 * j + 2;
        const bool next0 = j + 1 < qi.n_kv[0];
        const bool next1 = j + 1 < qi.n_kv[1];
        if (lane == 0) FA_TRACE_AT(j, 6);
        if (!(ok = wait(bar(L::kBarFull + slot_of(item_v)), phase_of(item_v), 12))) break;
        if ((next0 || next1) &&
            !(ok = wait(bar(L::kBarFull + slot_of(item_k)), phase_of(item_k), 14)))
          break;
        if (lane == 0) FA_TRACE_AT(j, 7);
        ptx::tc_fence_after();
        if (j < qi.n_kv[0]) {
          if (lane == 0) FA_TRACE_AT(j, 0);
          if (!(ok = issue_pv(0, item_v, j == 0, j & 1))) break;
          if (next0) {
            if (lane == 0) FA_TRACE_AT(j, 1);
            issue_s(0, item_k, q_desc0);
            if (!next1) commit(bar(L::kBarEmpty + slot_of(item_k)));
          }
        }
        if (j < qi.n_kv[1]) {
          if (lane == 0) FA_TRACE_AT(j, 2);
          if (!(ok = issue_pv(1, item_v, j == 0, j & 1))) break;
        }
        commit(bar(L::kBarEmpty + slot_of(item_v)));
        if (next1) {
          if (lane == 0) FA_TRACE_AT(j, 3);
          issue_s(1, item_k, q_desc1);
          commit(bar(L::kBarEmpty + slot_of(item_k)));
        }
      }
      // drain: every product completes before the pair's tensor memory is freed
      if (ptx::elect_one()) ptx::mma_commit_pair(bar(L::kBarDrain), 0x1);
      __syncwarp();
      bar_wait(bar(L::kBarDrain), 0, wc, 19, false);
      __syncwarp();
    }
  } else {
    // ================================================= softmax groups
    ptx::setmaxnreg_inc<kRegsSoftmax>();
    const Quad qi = decode_quad(p, p.item0 + static_cast<int>(blockIdx.x >> 1));
    const int g = warp >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + L::tS(g);
    const uint32_t tP = tmem + lane_off + L::tP(g);
    const uint32_t tO = tmem + lane_off + L::tO(g);
    const float sl = p.scale_log2;
    // P announcements go to CTA 0's barriers
    const uint32_t bar_p = leader ? bar(L::kBarP + g) : lead_bar(L::kBarP + g);
    const uint32_t bar_ph = leader ? bar(L::kBarPH + g) : lead_bar(L::kBarPH + g);
    // CTA 0 arrives locally, CTA 1 on CTA 0's barrier; P itself is ordered by
    // tcgen05.wait::st and the fence before the arrive and the MMA warp's
    // fence after its wait
    auto arrive = [leader](uint32_t b) {
      if (leader)
        ptx::mbar_arrive(b);
      else
        ptx::mbar_arrive_remote(b);
    };
    const int n_tiles = qi.n_kv[g];
    const int tile = 4 * qi.quad + 2 * g + static_cast<int>(rank);
    const int q_row = tile * kBlockM + r;
    const int nq = p.Nq, nk = p.Nk;
    int row_end = nk;
    int tile_end = nk;
    if (p.causal) {
      row_end = min(row_end, q_row % p.pos_mod + p.causal_off + 1);
      const int lo = tile * kBlockM;
      const int hi = min(lo + kBlockM - 1, nq - 1);
      const int min_pos = (p.pos_mod >= nq) ? lo
                          : (hi / p.pos_mod != lo / p.pos_mod) ? 0
                                                                : lo % p.pos_mod;
      tile_end = min(tile_end, min_pos + p.causal_off + 1);
    }
    bool ok = true;
    float m = -INFINITY;
    float l = 0.f;
    for (int j = 0; ok && j < n_tiles; ++j) {
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + g), j & 1, wc, 20 + g));
      if (!ok) break;
      if (lane == 0) FA_TRACE_AT(j, 16 + warp);
      ptx::tc_fence_after();
      float x[kBlockN];
      {
        uint32_t u0[32], u1[32], u2[32], u3[32];
        ptx::tmem_ld32(tS + 0, u0);
        ptx::tmem_ld32(tS + 32, u1);
        ptx::tmem_ld32(tS + 64, u2);
        ptx::tmem_ld32(tS + 96, u3);
        ptx::tmem_wait_ld();
        pin_after_wait<32>(u0);
        pin_after_wait<32>(u1);
        pin_after_wait<32>(u2);
        pin_after_wait<32>(u3);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          x[c] = __uint_as_float(u0[c]);
          x[32 + c] = __uint_as_float(u1[c]);
          x[64 + c] = __uint_as_float(u2[c]);
          x[96 + c] = __uint_as_float(u3[c]);
        }
      }
      const int key0 = j * kBlockN;
      const bool masked = key0 + kBlockN > tile_end;
      float m_tile;
      float sl_eff = sl;
      if (masked) {
        const int lim = row_end - key0;
#pragma unroll
        for (int c = 0; c < kBlockN; c += 2) ptx::fmul2(x[c], x[c + 1], x[c], x[c + 1], sl, sl);
#pragma unroll
        for (int c = 0; c < kBlockN; ++c)
          if (c >= lim) x[c] = -INFINITY;
        m_tile = row_extreme<kBlockN, false>(x);
        sl_eff = 1.0f;
      } else if (sl >= 0.f) {
        m_tile = row_extreme<kBlockN, false>(x) * sl;
      } else {
        m_tile = row_extreme<kBlockN, true>(x) * sl;
      }
      if (r == 0) FA_TRACE_AT(j, 28 + g);
      const float m_new = fmaxf(m, m_tile);
      const bool grow = m_new > m + kRescaleThreshold;
      if (j == 0) {
        m = m_new;
      } else {
        // O_g holds PV of tiles < j: their products completed before S_g(j)
        // was signalled (one issuing thread, in-order products)
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? ptx::ex2_approx(m - m_new) : 1.0f;
          // 8 columns at a time: the scores stay live in registers meanwhile
#pragma unroll 1
          for (int c = 0; c < D / 8; ++c) {
            uint32_t o[8];
            ptx::tmem_ld8(tO + c * 8, o);
            ptx::tmem_wait_ld();
            pin_after_wait<8>(o);
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              float a0 = __uint_as_float(o[i]), a1 = __uint_as_float(o[i + 1]);
              ptx::fmul2(a0, a1, a0, a1, alpha, alpha);
              o[i] = __float_as_uint(a0);
              o[i + 1] = __float_as_uint(a1);
            }
            ptx::tmem_st8(tO + c * 8, o);
          }
          ptx::tmem_wait_st();
          if (grow) l *= alpha;
        }
        if (grow) m = m_new;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      // P = exp2(x * sl_eff - m) into TMEM in quarters; the first
      // kPEarlyQuarters are announced on CTA 0's PH barrier once stored
      auto announce = [arrive, bar_ph] { arrive(bar_ph); };
      const float tile_sum = masked ? exp_tile<BF16, false>(x, sl_eff, neg_m, tP, announce)
                                    : exp_tile<BF16, true>(x, sl_eff, neg_m, tP, announce);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      if (lane == 0) FA_TRACE_AT(j, 8 + warp);
      arrive(bar_p);
      l += tile_sum;
    }

    // ---- epilogue: O / l -> global, LSE
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    const bool row_ok = q_row < nq;
    const long long lse_index = static_cast<long long>(qi.bh) * p.Nq + q_row;
    T* const orow = reinterpret_cast<T*>(p.o) + lse_index * D;
    if (n_tiles == 0) {
      if (row_ok) {
        uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
        if (p.lse != nullptr) p.lse[lse_index] = -INFINITY;
      }
    } else {
      if (ok)
        ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarO + g), (n_tiles - 1) & 1, wc, 22 + g));
      if (ok) {
        ptx::tc_fence_after();
        const float inv_l = (l > 0.f) ? 1.0f / l : 0.f;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        const float lse_row = (l > 0.f) ? (m_use + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          ptx::tmem_ld32(tO + c * 32, o);
          ptx::tmem_wait_ld();
          pin_after_wait<32>(o);
          uint32_t hv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            hv[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
          }
        }
        if (row_ok && p.lse != nullptr) p.lse[lse_index] = lse_row;
      }
    }
  }

  // ---- teardown: this CTA is done with its barriers, copies and tensor
  // memory; tell the other CTA, and free the pair's tensor memory once it
  // has said the same (CTA 0 has drained every product by now)
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    ptx::mbar_arrive_cluster(ptx::mapa(bar(L::kBarExit), rank ^ 1u));
    bar_wait_cluster(bar(L::kBarExit), 0, wc, 25, false);
  }
  __syncthreads();
  if (warp == kWarpMma) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, L::kTmemCols);
  }
}

}  // namespace pair2
