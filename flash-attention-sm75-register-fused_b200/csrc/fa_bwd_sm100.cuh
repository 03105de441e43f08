// Attention backward for B200 (sm_100a); included by fa_fwd_sm100.cu, whose
// helpers (bounded mbarrier waits, the device status word, pack2) it uses.
//
// With P = exp(S*scale - LSE), S = Q K^T and D_i = sum_c dO_ic O_ic:
//   dV = P^T dO,   dP = dO V^T,   dS = P * (dP - D),   dK = scale dS^T Q,
//   dQ = scale dS K
// (the FlashAttention-2 backward; the forward it differentiates follows
// src/reference/attention_ref.py:10-45).  The reference has no backward: its
// autograd Function raises (src/flash_attention_sm75/ops.py:47-52).
//
// Three kernels:
//   fa_bwd_prep_kernel  D and LSE*log2(e) per query row, padded to whole tiles
//   fa_bwd_dkdv_kernel  one CTA per (batch, KV head, 128-key tile): loops over
//                       the group's query heads and query tiles, S^T = K Q^T and
//                       dP^T = V dO^T on tcgen05, P^T and dS^T in registers,
//                       dV += P^T dO and dK += dS^T Q accumulated in TMEM
//   fa_bwd_dq_kernel    one CTA per (batch, query head, 128-query tile):
//                       S = Q K^T, dP = dO V^T, dS, dQ += dS K in TMEM
// S and dP are recomputed by both main kernels, so no atomics are needed (GQA
// groups accumulate dK / dV inside one CTA).
//
// Warps (256 threads): 0-3 elementwise (one TMEM lane = one row each),
// 4 TMA producer, 5 MMA issuer + TMEM owner, 6-7 idle.
// TMEM (512 columns): S 0..127 (its first 64 columns then hold P or dS as
// f16 pairs), dP 128..255 (dS^T in 128..191), accumulators at 256 and 256+d.

namespace fa {
namespace {

constexpr int kBwdThreads = 256;
constexpr int kBwdWarpLoad = 4;
constexpr int kBwdWarpMma = 5;

template <int D>
struct BwdLayout {
  static constexpr int kColBlocks = D / 64;
  static constexpr int kBlockBytes = 128 * 128;  // one 64-column block of a 128-row tile
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kSlots = (D == 128) ? 4 : 8;
  static constexpr int kVec = 128 * 4;  // one tile's LSE*log2e or D values
  static constexpr int kOffFix = 0;     // the CTA's two fixed tiles
  static constexpr int kOffRing = 2 * kTile;
  static constexpr int kOffVec = kOffRing + kSlots * kTile;  // vector of ring slot s
  static constexpr int kOffBar = kOffVec + kSlots * kVec;
  static constexpr int kBarFix = 0;
  static constexpr int kBarFull = 1;
  static constexpr int kBarEmpty = kBarFull + kSlots;
  // S and dP (or S^T, dP^T) computed: one barrier per half of the step's 128
  // queries in the dK/dV kernel (kBarS + h), one (kBarS) in the dQ kernel
  static constexpr int kBarS = kBarEmpty + kSlots;
  static constexpr int kBarP = kBarS + 2;            // P / dS written (128 arrivals), per half
  static constexpr int kBarG = kBarP + 2;            // all gradient MMAs completed
  static constexpr int kNumBars = kBarG + 1;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kDynBytes = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t tS = 0, tDP = 128, tAcc0 = 256, tAcc1 = 256 + D;
  static_assert(kDynBytes <= 227 * 1024, "shared memory budget");
};

// D_r = sum_c dO[r][c] O[r][c] and L2_r = LSE_r * log2(e) for every padded row
// r < n_pad of every (batch, query head); rows >= N get D = 0, L2 = +inf so that
// their P is exactly 0.  One warp per row.
template <bool BF16>
__global__ void __launch_bounds__(256) fa_bwd_prep_kernel(const void* __restrict__ o,
                                                          const void* __restrict__ dout,
                                                          const float* __restrict__ lse,
                                                          float* __restrict__ l2,
                                                          float* __restrict__ dd, int N, int n_pad,
                                                          long long n_rows, int d) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int lane = threadIdx.x & 31;
  const long long bh = row / n_pad;
  const int r = static_cast<int>(row % n_pad);
  float acc = 0.f;
  if (r < N) {
    const T* op = reinterpret_cast<const T*>(o) + (bh * N + r) * d;
    const T* gp = reinterpret_cast<const T*>(dout) + (bh * N + r) * d;
    for (int c = lane * 2; c < d; c += 64) {
      float2 a, g;
      if constexpr (BF16) {
        a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(op + c));
        g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gp + c));
      } else {
        a = __half22float2(*reinterpret_cast<const __half2*>(op + c));
        g = __half22float2(*reinterpret_cast<const __half2*>(gp + c));
      }
      acc = fmaf(a.x, g.x, fmaf(a.y, g.y, acc));
    }
  }
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
  if (lane == 0) {
    dd[row] = acc;
    l2[row] = (r < N) ? lse[bh * N + r] * 1.4426950408889634f : INFINITY;
  }
}

// Shared start-up of the two main kernels: aligned shared memory, barriers,
// TMEM.  Returns false (after recording an error) when the aligned layout
// does not fit or the launch already failed elsewhere.
template <typename L>
__device__ __forceinline__ bool bwd_setup(uint8_t* smem_raw, uint8_t*& smem, uint32_t& sbase,
                                          unsigned epoch, volatile int*& abort_flag,
                                          uint32_t& tmem, int warp) {
  smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                    ~static_cast<uintptr_t>(1023));
  if (static_cast<int>(smem - smem_raw) + L::kBytes > L::kDynBytes) {
    if (threadIdx.x == 0) record_error(epoch, FA_ERR_LAUNCH);
    return false;
  }
  sbase = ptx::smem_u32(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  if (threadIdx.x == 0) {
    const unsigned long long st = *reinterpret_cast<volatile unsigned long long*>(&g_fa_status);
    *abort_flag = ((st >> 32) == epoch && (st & 0xffffffffull) != 0ull) ? 1 : 0;
    for (int i = 0; i < L::kNumBars; ++i)
      ptx::mbar_init(sbase + L::kOffBar + 8u * i, (i == L::kBarP || i == L::kBarP + 1) ? 128u : 1u);
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (*abort_flag) return false;
  if (warp == kBwdWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), L::kTmemCols);
    ptx::tmem_relinquish();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();
  tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  return true;
}

template <typename L>
__device__ __forceinline__ void bwd_teardown(uint32_t tmem, int warp) {
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kBwdWarpMma) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, L::kTmemCols);
  }
}

// 128-row slab of a d-column fp32 TMEM accumulator (this thread's row) times
// `mul`, rounded to f16/bf16 and stored to row `dst` when `store`.
template <int D, bool BF16>
__device__ __forceinline__ void bwd_store_row(uint32_t t_acc, float mul, void* dst, bool store) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    uint32_t v[32];
    ptx::tmem_ld32(t_acc + c * 32, v);
    ptx::tmem_wait_ld();
    pin_after_wait<32>(v);
    uint32_t h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      h[i] = pack2<BF16>(__uint_as_float(v[2 * i]) * mul, __uint_as_float(v[2 * i + 1]) * mul);
    if (store) {
      uint4* out = reinterpret_cast<uint4*>(reinterpret_cast<T*>(dst) + c * 32);
#pragma unroll
      for (int i = 0; i < 4; ++i) out[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
    }
  }
}

// ------------------------------------------------------------------ dK, dV
template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1) fa_bwd_dkdv_kernel(const __grid_constant__ BwdParams p) {
  using L = BwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* smem;
  uint32_t sbase, tmem;
  volatile int* abort_flag;
  if (!bwd_setup<L>(smem_raw, smem, sbase, p.epoch, abort_flag, tmem, warp)) return;
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};

  // work: key tile t of KV head (b, hk); steps over the group's query heads
  // and the query tiles that see the key tile (causal: i >= t, heaviest first)
  const int t = blockIdx.x % p.n_tiles;
  const int bhk = blockIdx.x / p.n_tiles;
  const int b = bhk / p.Hkv;
  const int hk = bhk % p.Hkv;
  const int i0 = p.causal ? t : 0;
  const int n_q = p.n_tiles - i0;
  const int n_steps = p.group * n_q;
  auto step_head = [&](int s) { return b * p.Hq + hk * p.group + s / n_q; };  // b*Hq + h
  auto step_tile = [&](int s) { return i0 + s % n_q; };

  if (warp == kBwdWarpLoad) {
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_last();
      ptx::mbar_arrive_expect_tx(bar(L::kBarFix), 2 * L::kTile);
#pragma unroll
      for (int c = 0; c < L::kColBlocks; ++c) {
        ptx::tma_load_3d(sbase + L::kOffFix + c * L::kBlockBytes, &p.tm_k, bar(L::kBarFix), c * 64,
                         t * 128, bhk, pol);
        ptx::tma_load_3d(sbase + L::kOffFix + L::kTile + c * L::kBlockBytes, &p.tm_v,
                         bar(L::kBarFix), c * 64, t * 128, bhk, pol);
      }
      // ring item 2s: Q tile (+ its L2 vector), 2s+1: dO tile (+ its D vector)
      int issued = 0;
      for (int i = 0; i < 2 * n_steps; ++i) {
        const int slot = i % L::kSlots;
        if (i >= L::kSlots && !bar_wait(bar(L::kBarEmpty + slot), ((i / L::kSlots) - 1) & 1, wc, 41))
          break;
        const int s = i >> 1;
        const int bhq = step_head(s);
        const int qt = step_tile(s);
        const void* map = (i & 1) ? static_cast<const void*>(&p.tm_do) : static_cast<const void*>(&p.tm_q);
        const float* vec = ((i & 1) ? p.dd : p.l2) + static_cast<size_t>(bhq) * p.n_pad + qt * 128;
        ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile + L::kVec);
#pragma unroll
        for (int c = 0; c < L::kColBlocks; ++c)
          ptx::tma_load_3d(sbase + L::kOffRing + slot * L::kTile + c * L::kBlockBytes, map,
                           bar(L::kBarFull + slot), c * 64, qt * 128, bhq, pol);
        ptx::bulk_load(sbase + L::kOffVec + slot * L::kVec, vec, L::kVec, bar(L::kBarFull + slot));
        issued = i + 1;
      }
      for (int i = max(0, issued - L::kSlots); i < issued; ++i)
        bar_wait(bar(L::kBarFull + i % L::kSlots), (i / L::kSlots) & 1, wc, 42, false);
      bar_wait(bar(L::kBarFix), 0, wc, 42, false);
    }
  } else if (warp == kBwdWarpMma) {
    // Each step's 128 queries are processed as two halves h of 64.  Issue
    // order: S(0,h0) dP(0,h0) S(0,h1) dP(0,h1), then per step s and half h
    //   [P(s,h) ready]  dV += P^T(s,h) dO(s,h)  dK += dS^T(s,h) Q(s,h)
    //                   S(s+1,h)  dP(s+1,h)
    // so the elementwise phase of one half runs while the tensor pipe works on
    // the other.  S(s+1,h) overwrites the TMEM columns holding P^T(s,h) and
    // dP(s+1,h) those holding dS^T(s,h); tcgen05.mma ops of one thread execute
    // in issue order, so the gradient products have read them first.
    constexpr uint32_t fmt = BF16 ? 1u : 0u;
    constexpr uint32_t idesc_s = ptx::make_idesc_f16(128, 64, fmt, 0, 0);
    constexpr uint32_t idesc_g = ptx::make_idesc_f16(128, D, fmt, 0, 1);
    auto slot_of = [](int i) { return i % L::kSlots; };
    auto phase_of = [](int i) { return static_cast<uint32_t>((i / L::kSlots) & 1); };
    auto wait = [&](uint32_t bb, uint32_t ph, int site) {
      return __all_sync(0xffffffffu, bar_wait(bb, ph, wc, site));
    };
    const uint64_t k_desc = ptx::smem_desc_sw128(sbase + L::kOffFix, 16, 1024);
    const uint64_t v_desc = ptx::smem_desc_sw128(sbase + L::kOffFix + L::kTile, 16, 1024);
    const uint64_t ring_k = ptx::smem_desc_sw128(sbase + L::kOffRing, 16, 1024);              // K-major
    const uint64_t ring_mn = ptx::smem_desc_sw128(sbase + L::kOffRing, L::kBlockBytes, 1024);  // MN-major
    // S^T(s,h) = K Q^T and dP^T(s,h) = V dO^T for queries [64h, 64h+64) of
    // step s (B = 64 rows of the Q / dO tile: 8 KB into each 64-column block)
    auto issue_scores = [&](int s, int h) {
      const uint64_t q_off = static_cast<uint64_t>((slot_of(2 * s) * L::kTile + h * 8192) >> 4);
      const uint64_t d_off = static_cast<uint64_t>((slot_of(2 * s + 1) * L::kTile + h * 8192) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
          ptx::mma_ss(tmem + L::tS + 64 * h, k_desc + off, ring_k + q_off + off, idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
          ptx::mma_ss(tmem + L::tDP + 64 * h, v_desc + off, ring_k + d_off + off, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(bar(L::kBarS + h));
      }
      __syncwarp();
    };
    // dV += P^T dO and dK += dS^T Q over queries [64h, 64h+64) of step s
    // (A from TMEM: P^T / dS^T packed in the half's first 32 columns; B
    // MN-major, K = queries, 16 rows = 2 KB per K step)
    auto issue_grads = [&](int s, int h) {
      const uint64_t q_off = static_cast<uint64_t>((slot_of(2 * s) * L::kTile) >> 4);
      const uint64_t d_off = static_cast<uint64_t>((slot_of(2 * s + 1) * L::kTile) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t off = static_cast<uint64_t>(((4 * h + k) * 2048) >> 4);
          ptx::mma_ts(tmem + L::tAcc0, tmem + L::tS + 64 * h + 8 * k, ring_mn + d_off + off, idesc_g,
                      (s > 0 || h > 0 || k > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t off = static_cast<uint64_t>(((4 * h + k) * 2048) >> 4);
          ptx::mma_ts(tmem + L::tAcc1, tmem + L::tDP + 64 * h + 8 * k, ring_mn + q_off + off, idesc_g,
                      (s > 0 || h > 0 || k > 0) ? 1u : 0u);
        }
        if (h == 1) {  // the step's Q and dO tiles are read for the last time
          ptx::mma_commit(bar(L::kBarEmpty + slot_of(2 * s)));
          ptx::mma_commit(bar(L::kBarEmpty + slot_of(2 * s + 1)));
        }
      }
      __syncwarp();
    };
    bool ok = wait(bar(L::kBarFix), 0, 43);
    if (ok && n_steps > 0) {
      ok = wait(bar(L::kBarFull + slot_of(0)), phase_of(0), 44) &&
           wait(bar(L::kBarFull + slot_of(1)), phase_of(1), 44);
      if (ok) {
        ptx::tc_fence_after();
        issue_scores(0, 0);
        issue_scores(0, 1);
      }
    }
    for (int s = 0; ok && s < n_steps; ++s) {
      const bool next = s + 1 < n_steps;
      if (next) {
        const int iq = 2 * s + 2, id = 2 * s + 3;
        if (!(ok = wait(bar(L::kBarFull + slot_of(iq)), phase_of(iq), 44))) break;
        if (!(ok = wait(bar(L::kBarFull + slot_of(id)), phase_of(id), 44))) break;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!(ok = wait(bar(L::kBarP + h), s & 1, 45))) break;
        ptx::tc_fence_after();
        issue_grads(s, h);
        if (next) issue_scores(s + 1, h);
      }
    }
    if (ptx::elect_one()) ptx::mma_commit(bar(L::kBarG));
    __syncwarp();
    bar_wait(bar(L::kBarG), 0, wc, 46, false);
    __syncwarp();
  } else if (warp < 4) {
    // rows = keys of tile t; columns = the step's 128 queries, in two halves
    const int r = warp * 32 + lane;
    const int key = t * 128 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float sl = p.scale_log2;
    bool ok = true;
    for (int s = 0; ok && s < n_steps; ++s) {
      const int qt = step_tile(s);
      const float4* l2v = reinterpret_cast<const float4*>(smem + L::kOffVec + ((2 * s) % L::kSlots) * L::kVec);
      const float4* ddv = reinterpret_cast<const float4*>(smem + L::kOffVec + ((2 * s + 1) % L::kSlots) * L::kVec);
      const bool diag = p.causal && qt == t;  // query < key is masked
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + h), s & 1, wc, 47));
        if (!ok) break;
        ptx::tc_fence_after();
        uint32_t pk[32], gk[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t sv[32], dv[32];
          ptx::tmem_ld32(tmem + lane_off + L::tS + 64 * h + 32 * c, sv);
          ptx::tmem_ld32(tmem + lane_off + L::tDP + 64 * h + 32 * c, dv);
          ptx::tmem_wait_ld();
          pin_after_wait<32>(sv);
          pin_after_wait<32>(dv);
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const int q0 = 64 * h + 32 * c + i;  // query within the tile
            const float4 lv = l2v[q0 / 4];
            const float4 dd = ddv[q0 / 4];
            const float lq[4] = {lv.x, lv.y, lv.z, lv.w};
            const float dq[4] = {dd.x, dd.y, dd.z, dd.w};
            float pe[4], ge[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float pv = ptx::ex2_approx(fmaf(__uint_as_float(sv[i + e]), sl, -lq[e]));
              if (diag && q0 + e < r) pv = 0.f;
              pe[e] = pv;
              ge[e] = pv * (__uint_as_float(dv[i + e]) - dq[e]);
            }
            pk[16 * c + i / 2] = pack2<BF16>(pe[0], pe[1]);
            pk[16 * c + i / 2 + 1] = pack2<BF16>(pe[2], pe[3]);
            gk[16 * c + i / 2] = pack2<BF16>(ge[0], ge[1]);
            gk[16 * c + i / 2 + 1] = pack2<BF16>(ge[2], ge[3]);
          }
        }
        // P^T into S columns 64h.., dS^T into dP columns 64h.. (both already read)
        ptx::tmem_st32(tmem + lane_off + L::tS + 64 * h, pk);
        ptx::tmem_st32(tmem + lane_off + L::tDP + 64 * h, gk);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(L::kBarP + h));
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarG), 0, wc, 48));
    if (ok) {
      ptx::tc_fence_after();
      const bool store = key < p.N;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      const size_t row = static_cast<size_t>(bhk) * p.N + key;
      bwd_store_row<D, BF16>(tmem + lane_off + L::tAcc0, 1.0f, reinterpret_cast<T*>(p.dv) + row * D, store);
      bwd_store_row<D, BF16>(tmem + lane_off + L::tAcc1, p.scale, reinterpret_cast<T*>(p.dk) + row * D, store);
    }
  }
  bwd_teardown<L>(tmem, warp);
}

// ------------------------------------------------------------------ dQ
template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1) fa_bwd_dq_kernel(const __grid_constant__ BwdParams p) {
  using L = BwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* smem;
  uint32_t sbase, tmem;
  volatile int* abort_flag;
  if (!bwd_setup<L>(smem_raw, smem, sbase, p.epoch, abort_flag, tmem, warp)) return;
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};

  // work: query tile t of (b, hq); key tiles 0..n_kv-1 (causal: j <= t,
  // heaviest tiles first)
  int t = blockIdx.x % p.n_tiles;
  if (p.causal) t = p.n_tiles - 1 - t;
  const int bh = blockIdx.x / p.n_tiles;
  const int b = bh / p.Hq;
  const int bh_kv = b * p.Hkv + (bh % p.Hq) / p.group;
  const int n_kv = p.causal ? t + 1 : p.n_tiles;

  if (warp == kBwdWarpLoad) {
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_last();
      ptx::mbar_arrive_expect_tx(bar(L::kBarFix), 2 * L::kTile);
#pragma unroll
      for (int c = 0; c < L::kColBlocks; ++c) {
        ptx::tma_load_3d(sbase + L::kOffFix + c * L::kBlockBytes, &p.tm_q, bar(L::kBarFix), c * 64,
                         t * 128, bh, pol);
        ptx::tma_load_3d(sbase + L::kOffFix + L::kTile + c * L::kBlockBytes, &p.tm_do,
                         bar(L::kBarFix), c * 64, t * 128, bh, pol);
      }
      // ring item 2j: K_j, 2j+1: V_j
      int issued = 0;
      for (int i = 0; i < 2 * n_kv; ++i) {
        const int slot = i % L::kSlots;
        if (i >= L::kSlots && !bar_wait(bar(L::kBarEmpty + slot), ((i / L::kSlots) - 1) & 1, wc, 51))
          break;
        const void* map = (i & 1) ? static_cast<const void*>(&p.tm_v) : static_cast<const void*>(&p.tm_k);
        ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile);
#pragma unroll
        for (int c = 0; c < L::kColBlocks; ++c)
          ptx::tma_load_3d(sbase + L::kOffRing + slot * L::kTile + c * L::kBlockBytes, map,
                           bar(L::kBarFull + slot), c * 64, (i >> 1) * 128, bh_kv, pol);
        issued = i + 1;
      }
      for (int i = max(0, issued - L::kSlots); i < issued; ++i)
        bar_wait(bar(L::kBarFull + i % L::kSlots), (i / L::kSlots) & 1, wc, 52, false);
      bar_wait(bar(L::kBarFix), 0, wc, 52, false);
    }
  } else if (warp == kBwdWarpMma) {
    // Keys of each K/V tile in two halves h of 64, issued as
    //   S(0,h0) dP(0,h0) S(0,h1) dP(0,h1), then per tile j and half h:
    //   [dS(j,h) ready]  dQ += dS(j,h) K(j,h)  S(j+1,h)  dP(j+1,h)
    // (the elementwise phase of one half overlaps the other half's products;
    // S(j+1,h) overwrites the columns of dS(j,h) after dQ has read them, in
    // issue order).
    constexpr uint32_t fmt = BF16 ? 1u : 0u;
    constexpr uint32_t idesc_s = ptx::make_idesc_f16(128, 64, fmt, 0, 0);
    constexpr uint32_t idesc_g = ptx::make_idesc_f16(128, D, fmt, 0, 1);
    auto slot_of = [](int i) { return i % L::kSlots; };
    auto phase_of = [](int i) { return static_cast<uint32_t>((i / L::kSlots) & 1); };
    auto wait = [&](uint32_t bb, uint32_t ph, int site) {
      return __all_sync(0xffffffffu, bar_wait(bb, ph, wc, site));
    };
    const uint64_t q_desc = ptx::smem_desc_sw128(sbase + L::kOffFix, 16, 1024);
    const uint64_t do_desc = ptx::smem_desc_sw128(sbase + L::kOffFix + L::kTile, 16, 1024);
    const uint64_t ring_k = ptx::smem_desc_sw128(sbase + L::kOffRing, 16, 1024);
    const uint64_t ring_mn = ptx::smem_desc_sw128(sbase + L::kOffRing, L::kBlockBytes, 1024);
    // S(j,h) = Q K^T, dP(j,h) = dO V^T over keys [64h, 64h+64) of tile j
    auto issue_scores = [&](int j, int h) {
      const uint64_t k_off = static_cast<uint64_t>((slot_of(2 * j) * L::kTile + h * 8192) >> 4);
      const uint64_t v_off = static_cast<uint64_t>((slot_of(2 * j + 1) * L::kTile + h * 8192) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
          ptx::mma_ss(tmem + L::tS + 64 * h, q_desc + off, ring_k + k_off + off, idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
          ptx::mma_ss(tmem + L::tDP + 64 * h, do_desc + off, ring_k + v_off + off, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(bar(L::kBarS + h));
        if (h == 1) ptx::mma_commit(bar(L::kBarEmpty + slot_of(2 * j + 1)));  // V_j read
      }
      __syncwarp();
    };
    // dQ += dS(j,h) K(j,h) (A = dS from TMEM, B = K_j MN-major: K = keys)
    auto issue_grad = [&](int j, int h) {
      const uint64_t k_off = static_cast<uint64_t>((slot_of(2 * j) * L::kTile) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t off = static_cast<uint64_t>(((4 * h + k) * 2048) >> 4);
          ptx::mma_ts(tmem + L::tAcc0, tmem + L::tS + 64 * h + 8 * k, ring_mn + k_off + off, idesc_g,
                      (j > 0 || h > 0 || k > 0) ? 1u : 0u);
        }
        if (h == 1) ptx::mma_commit(bar(L::kBarEmpty + slot_of(2 * j)));  // K_j read
      }
      __syncwarp();
    };
    bool ok = wait(bar(L::kBarFix), 0, 53);
    if (ok && n_kv > 0) {
      ok = wait(bar(L::kBarFull + slot_of(0)), phase_of(0), 54) &&
           wait(bar(L::kBarFull + slot_of(1)), phase_of(1), 54);
      if (ok) {
        ptx::tc_fence_after();
        issue_scores(0, 0);
        issue_scores(0, 1);
      }
    }
    for (int j = 0; ok && j < n_kv; ++j) {
      const bool next = j + 1 < n_kv;
      if (next) {
        const int ik = 2 * j + 2, iv = 2 * j + 3;
        if (!(ok = wait(bar(L::kBarFull + slot_of(ik)), phase_of(ik), 54))) break;
        if (!(ok = wait(bar(L::kBarFull + slot_of(iv)), phase_of(iv), 54))) break;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!(ok = wait(bar(L::kBarP + h), j & 1, 55))) break;
        ptx::tc_fence_after();
        issue_grad(j, h);
        if (next) issue_scores(j + 1, h);
      }
    }
    if (ptx::elect_one()) ptx::mma_commit(bar(L::kBarG));
    __syncwarp();
    bar_wait(bar(L::kBarG), 0, wc, 56, false);
    __syncwarp();
  } else if (warp < 4) {
    const int r = warp * 32 + lane;
    const int q_row = t * 128 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float sl = p.scale_log2;
    const float lv = p.l2[static_cast<size_t>(bh) * p.n_pad + q_row];
    const float dval = p.dd[static_cast<size_t>(bh) * p.n_pad + q_row];
    bool ok = true;
    for (int j = 0; ok && j < n_kv; ++j) {
      // keys >= N and (causal) keys > this query get P = 0
      int lim = p.N - j * 128;
      if (p.causal && j == t) lim = min(lim, r + 1);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + h), j & 1, wc, 57));
        if (!ok) break;
        ptx::tc_fence_after();
        uint32_t gk[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t sv[32], dv[32];
          ptx::tmem_ld32(tmem + lane_off + L::tS + 64 * h + 32 * c, sv);
          ptx::tmem_ld32(tmem + lane_off + L::tDP + 64 * h + 32 * c, dv);
          ptx::tmem_wait_ld();
          pin_after_wait<32>(sv);
          pin_after_wait<32>(dv);
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float ge[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              float pv = ptx::ex2_approx(fmaf(__uint_as_float(sv[i + e]), sl, -lv));
              if (64 * h + 32 * c + i + e >= lim) pv = 0.f;
              ge[e] = pv * (__uint_as_float(dv[i + e]) - dval);
            }
            gk[16 * c + i / 2] = pack2<BF16>(ge[0], ge[1]);
          }
        }
        ptx::tmem_st32(tmem + lane_off + L::tS + 64 * h, gk);  // dS into S columns (read)
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(L::kBarP + h));
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarG), 0, wc, 58));
    if (ok) {
      ptx::tc_fence_after();
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      const size_t row = static_cast<size_t>(bh) * p.N + q_row;
      bwd_store_row<D, BF16>(tmem + lane_off + L::tAcc0, p.scale, reinterpret_cast<T*>(p.dq) + row * D,
                             q_row < p.N);
    }
  }
  bwd_teardown<L>(tmem, warp);
}

}  // namespace

template <int D, bool BF16>
static cudaError_t launch_bwd_impl(const BwdParams& p, const void* o, const void* dout,
                                   const float* lse, cudaStream_t stream) {
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fa_bwd_dkdv_kernel<D, BF16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         BwdLayout<D>::kDynBytes);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fa_bwd_dq_kernel<D, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               BwdLayout<D>::kDynBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  const long long rows = static_cast<long long>(p.B) * p.Hq * p.n_pad;
  fa_bwd_prep_kernel<BF16><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
      o, dout, lse, const_cast<float*>(p.l2), const_cast<float*>(p.dd), p.N, p.n_pad, rows, D);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  fa_bwd_dkdv_kernel<D, BF16><<<p.B * p.Hkv * p.n_tiles, kBwdThreads, BwdLayout<D>::kDynBytes, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  fa_bwd_dq_kernel<D, BF16><<<p.B * p.Hq * p.n_tiles, kBwdThreads, BwdLayout<D>::kDynBytes, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_bwd(const BwdParams& p, const void* o, const void* dout, const float* lse,
                       int head_dim, bool bf16, cudaStream_t stream) {
  if (head_dim == 64)
    return bf16 ? launch_bwd_impl<64, true>(p, o, dout, lse, stream)
                : launch_bwd_impl<64, false>(p, o, dout, lse, stream);
  return bf16 ? launch_bwd_impl<128, true>(p, o, dout, lse, stream)
              : launch_bwd_impl<128, false>(p, o, dout, lse, stream);
}

int bwd_smem_bytes_for(int head_dim) {
  return head_dim == 64 ? BwdLayout<64>::kDynBytes : BwdLayout<128>::kDynBytes;
}

}  // namespace fa
