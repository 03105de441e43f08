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
//   fa_bwd_prep_kernel  per query row -LSE*log2(e) and -D (padded to whole
//                       tiles), and per 128-row query tile two K-major operand
//                       tiles holding -LSE/scale and -D as 16-bit terms
//   fa_bwd_dkdv_kernel  one CTA per (batch, KV head, 128-key tile): loops over
//                       the group's query heads and query tiles; issue order
//                       dV += P^T(s) dO(s), S^T(s+1), dK += dS^T(s) Q(s),
//                       dP^T(s+1), the score products starting from a
//                       ones x vector product that pre-loads -LSE/scale (-D)
//   fa_bwd_dq_kernel    one CTA per (batch, query head, 128-query tile), Q in
//                       TMEM: S(j+1) = Q K^T as soon as S(j) is read, then
//                       dQ += dS(j) K_j and dP(j+1)
// S and dP are recomputed by both main kernels, so no atomics are needed (GQA
// groups accumulate dK / dV inside one CTA).
//
// Development builds (-DFA_TRACE) record clock64 timelines of the first
// CTAs into BwdParams::trace (dK/dV kernel: per step s, MMA warp events 1-5,
// elementwise warp 0 events 8-15, 17-18, producer event 16; dQ kernel: per
// K/V tile j, MMA warp events 19-23, elementwise warp 0 events 24-28).
//
// Warps (384 threads): 0-7 elementwise in two groups g (warps 4g..4g+3, one
// TMEM lane = one row per thread, columns [64g, 64g+64) of the 128), 8 TMA
// producer, 9 MMA issuer + TMEM owner, 10-11 idle.
// TMEM (512 columns), dK/dV kernel: S^T 0..127, dP^T 128..255, dV and dK
// accumulators at 256 and 256+d; group g packs its P^T / dS^T (f16 pairs)
// into the first 32 of its own 64 S / dP columns.  dQ kernel: S, dP, the dQ
// accumulator at 256, packed dS at 256+d (group g: columns 32g..) and Q (the
// A operand of S) at 320+d.

namespace fa {
namespace {

constexpr int kBwdThreads = 384;
constexpr int kBwdWarpLoad = 8;
constexpr int kBwdWarpMma = 9;
constexpr int kBwdElemThreads = 256;  // warps 0-7: two groups of 64 columns each

template <int D>
struct BwdLayout {
  static constexpr int kColBlocks = D / 64;
  static constexpr int kBlockBytes = 128 * 128;  // one 64-column block of a 128-row tile
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kSlots = (D == 128) ? 4 : 8;
  // K-major 128x16 operand tile without swizzle (see BwdParams::vt)
  static constexpr int kVec = 4096;
  static constexpr int kOffFix = 0;     // the CTA's two fixed tiles
  static constexpr int kOffRing = 2 * kTile;
  static constexpr int kOffVec = kOffRing + kSlots * kTile;  // vector tile of ring slot s
  static constexpr int kOffOnes = kOffVec + kSlots * kVec;   // A operand: ones in k = 0..2
  static constexpr int kOffBar = kOffOnes + kVec;
  static constexpr int kBarFix = 0;
  static constexpr int kBarFull = 1;
  static constexpr int kBarEmpty = kBarFull + kSlots;
  // kBarS: S (S^T) computed; kBarS + 1: dP (dP^T) computed
  static constexpr int kBarS = kBarEmpty + kSlots;
  // 128 arrivals each.  dK/dV kernel: kBarP = P^T written, kBarP + 1 = dS^T
  // written.  dQ kernel: kBarP = S read, kBarP + 1 = dS written.
  static constexpr int kBarP = kBarS + 2;
  static constexpr int kBarG = kBarP + 2;            // all gradient MMAs completed
  static constexpr int kBarQT = kBarG + 1;           // dQ kernel: Q copied into TMEM (128 arrivals)
  static constexpr int kNumBars = kBarQT + 1;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kBytes = kOffMisc + 16;
  static constexpr int kDynBytes = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t tS = 0, tDP = 128, tAcc0 = 256, tAcc1 = 256 + D;
  static constexpr uint32_t tDS = 256 + D;       // dQ kernel: packed dS (64 columns)
  static constexpr uint32_t tQ = 256 + D + 64;   // dQ kernel: Q as the A operand (d/2 columns)
  static_assert(tQ + D / 2 <= kTmemCols, "tensor memory budget");
  static_assert(kDynBytes <= 227 * 1024, "shared memory budget");
};

// First row and length of batch entry b's sequence: the packed varlen layout
// reads them from cu_seqlens (clamped to the tensors), the fixed layout has
// every sequence at rows [0, N).
// Block -> (tile, head) of the two main kernels.  Non-causal: head-major.
// Causal tiles differ in work (a factor of n_tiles): blocks go tile-major
// within groups of kBwdHeadGroup heads and head-major across groups, so each
// group starts its heaviest tiles first while the CTAs that run together
// still share a few heads' tensors in L2 (fully tile-major order measured
// 23 % slower on a causal C5 backward).  `t` counts from the heavy end.
constexpr int kBwdHeadGroup = 4;  // groups of 4 and 8 heads measured alike
__device__ __forceinline__ void bwd_block_order(int causal, int block, int n_heads, int n_tiles,
                                                int& t, int& head) {
  if (!causal) {
    t = block % n_tiles;
    head = block / n_tiles;
    return;
  }
  const int per_group = kBwdHeadGroup * n_tiles;
  const int g = block / per_group;
  const int r = block % per_group;
  const int g_heads = min(kBwdHeadGroup, n_heads - g * kBwdHeadGroup);
  t = r / g_heads;
  head = g * kBwdHeadGroup + r % g_heads;
}

__device__ __forceinline__ void bwd_seq(const int* cu, int total, int N, int b, int& start,
                                        int& n) {
  if (cu == nullptr) {
    start = 0;
    n = N;
    return;
  }
  start = min(max(__ldg(cu + b), 0), total);
  n = min(min(max(__ldg(cu + b + 1), start), total) - start, N);
}

// Per padded row r < n_pad of every (batch, query head): nl2_r = -LSE_r*log2(e)
// and nd_r = -D_r = -sum_c dO[r][c] O[r][c] (negated so that the main kernels
// form s*scale*log2(e) - LSE*log2(e) and dP - D with one packed FMA / add);
// rows >= N get nl2 = -inf, nd = 0, so their P is 0.  d/8 lanes per row, each
// reading 16 bytes of O and of dO (the kernel streams O and dO once).
template <bool BF16>
__global__ void __launch_bounds__(256) fa_bwd_prep_kernel(const void* __restrict__ o,
                                                          const void* __restrict__ dout,
                                                          const float* __restrict__ lse,
                                                          float* __restrict__ l2,
                                                          float* __restrict__ dd,
                                                          uint8_t* __restrict__ vt, float scale,
                                                          int N, int n_pad, long long n_rows,
                                                          int d, int heads,
                                                          const int* __restrict__ q_lo,
                                                          const int* __restrict__ q_hi,
                                                          const int* __restrict__ cu, int total) {
  const int lpr = d >> 3;  // lanes per row: 16 (d = 128) or 8 (d = 64)
  const int rows_per_block = 256 / lpr;
  const long long row = static_cast<long long>(blockIdx.x) * rows_per_block + threadIdx.x / lpr;
  const int sub = threadIdx.x % lpr;
  const bool live = row < n_rows;
  const long long bh = live ? row / n_pad : 0;
  const int r = live ? static_cast<int>(row % n_pad) : N;
  // a row outside its batch entry's query range or sequence, or one that saw
  // no key (LSE = -inf), is treated like a padded row: P = 0
  const int b = static_cast<int>(bh / heads), h = static_cast<int>(bh % heads);
  int start, n;
  bwd_seq(cu, total, N, b, start, n);
  bool valid = live && r < n;
  if (valid && q_lo != nullptr) valid = r >= __ldg(q_lo + b) && r < __ldg(q_hi + b);
  // element offset of the row in O / dO and its LSE index (packed: [total, H, d], [H, total])
  const long long orow = cu ? (static_cast<long long>(start + r) * heads + h) * d : (bh * N + r) * d;
  const float lse_r = valid ? lse[cu ? static_cast<long long>(h) * total + start + r : bh * N + r] : 0.f;
  if (valid && lse_r == -INFINITY) valid = false;
  float acc = 0.f;
  if (valid) {
    const uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(o) +
                                                    (orow + sub * 8) * 2);
    const uint4 g = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(dout) +
                                                    (orow + sub * 8) * 2);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 fa, fg;
      if constexpr (BF16) {
        fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&av[i]));
        fg = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gv[i]));
      } else {
        fa = __half22float2(*reinterpret_cast<const __half2*>(&av[i]));
        fg = __half22float2(*reinterpret_cast<const __half2*>(&gv[i]));
      }
      acc = fmaf(fa.x, fg.x, fmaf(fa.y, fg.y, acc));
    }
  }
  // sum over the row's lanes (aligned groups of lpr lanes within the warp)
  for (int m = lpr >> 1; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  if (!live) return;
  const int lane = sub;
  if (lane == 0) {
    dd[row] = -acc;
    l2[row] = valid ? -lse_r * 1.4426950408889634f : -INFINITY;
    // operand tiles of the dK/dV kernel: -LSE/scale (a large negative value
    // for padded rows, whose P must vanish) and -D as three 16-bit terms
    const float vals[2] = {valid ? -lse_r / scale : -30000.f, -acc};
    const int n = r & 127;
    uint8_t* tile = vt + (static_cast<size_t>(row >> 7) * 2) * 4096 + (n >> 3) * 256 + (n & 7) * 16;
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      uint32_t h[3];
      float rest = vals[v];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        if constexpr (BF16) {
          const __nv_bfloat16 t = __float2bfloat16_rn(rest);
          rest -= __bfloat162float(t);
          h[k] = *reinterpret_cast<const unsigned short*>(&t);
        } else {
          const __half t = __float2half_rn(rest);
          rest -= __half2float(t);
          h[k] = *reinterpret_cast<const unsigned short*>(&t);
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(tile + v * 4096);
      dst[0] = make_uint4(h[0] | (h[1] << 16), h[2], 0u, 0u);  // k = 0..7
      dst[8] = make_uint4(0u, 0u, 0u, 0u);                     // k = 8..15 (128 B further)
    }
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
      ptx::mbar_init(sbase + L::kOffBar + 8u * i,
                     (i == L::kBarP || i == L::kBarP + 1) ? static_cast<uint32_t>(kBwdElemThreads)
                     : i == L::kBarQT                     ? 128u
                                                          : 1u);
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

// One in kBwdEmuEvery pairs of exponentials is evaluated by the FMA-pipe
// polynomial (exp2_poly2) instead of the MUFU unit, which is the elementwise
// phase's narrowest pipe.
#ifndef FA_BWD_EMU_EVERY
#define FA_BWD_EMU_EVERY 4
#endif
constexpr int kBwdEmuEvery = FA_BWD_EMU_EVERY;

// p[i] = 2^(s[i] * sl + nl[i]) for 32 scores of this thread's row, masked
// (MASK) to 0 outside lo <= i < hi.  nl holds 32 per-column values or, with
// nl_col == nullptr, one value for the row.
template <bool MASK>
__device__ __forceinline__ void bwd_exp32(float* p, const uint32_t (&sv)[32], float sl,
                                          const float4* nl_col, float nl_row, int lo, int hi) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    float4 nl;
    if (nl_col != nullptr) nl = nl_col[i / 4];
    else nl = make_float4(nl_row, nl_row, nl_row, nl_row);
    float t0, t1, t2, t3;
    ptx::ffma2(t0, t1, __uint_as_float(sv[i]), __uint_as_float(sv[i + 1]), sl, sl, nl.x, nl.y);
    ptx::ffma2(t2, t3, __uint_as_float(sv[i + 2]), __uint_as_float(sv[i + 3]), sl, sl, nl.z, nl.w);
    if ((i / 2) % kBwdEmuEvery == 0) {
      ptx::exp2_poly2(p[i], p[i + 1], t0, t1);
    } else {
      p[i] = ptx::ex2_approx(t0);
      p[i + 1] = ptx::ex2_approx(t1);
    }
    p[i + 2] = ptx::ex2_approx(t2);
    p[i + 3] = ptx::ex2_approx(t3);
    if (MASK) {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (i + e < lo || i + e >= hi) p[i + e] = 0.f;
    }
  }
}

// g = P * (dP + nd) (ADD) or P * dP, 32 values packed to f16/bf16 pairs; nd
// per column (nd_col) or one value (nd_col == nullptr).
template <bool BF16, bool ADD>
__device__ __forceinline__ void bwd_ds32(uint32_t (&gk)[16], const float* p,
                                         const uint32_t (&dv)[32], const float4* nd_col,
                                         float nd_row) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    float a0 = __uint_as_float(dv[i]), a1 = __uint_as_float(dv[i + 1]);
    float a2 = __uint_as_float(dv[i + 2]), a3 = __uint_as_float(dv[i + 3]);
    if (ADD) {
      float4 nd;
      if (nd_col != nullptr) nd = nd_col[i / 4];
      else nd = make_float4(nd_row, nd_row, nd_row, nd_row);
      ptx::fadd2(a0, a1, a0, a1, nd.x, nd.y);
      ptx::fadd2(a2, a3, a2, a3, nd.z, nd.w);
    }
    ptx::fmul2(a0, a1, a0, a1, p[i], p[i + 1]);
    ptx::fmul2(a2, a3, a2, a3, p[i + 2], p[i + 3]);
    gk[i / 2] = pack2<BF16>(a0, a1);
    gk[i / 2 + 1] = pack2<BF16>(a2, a3);
  }
}

// ------------------------------------------------------------------ dK, dV
template <int D, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1) fa_bwd_dkdv_kernel(const __grid_constant__ BwdParams p) {
  using L = BwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // work: key tile t of KV head (b, hk); steps over the group's query heads
  // and the query tiles that see the key tile (causal: i >= t, heaviest first
  // within each group of kBwdHeadGroup heads)
  int t, bhk;
  bwd_block_order(p.causal, static_cast<int>(blockIdx.x), p.B * p.Hkv, p.n_tiles, t, bhk);
  const int b = bhk / p.Hkv;
  const int hk = bhk % p.Hkv;
  int start, n;  // sequence of batch entry b (packed varlen: its rows)
  bwd_seq(p.cu, p.total, p.N, b, start, n);
  if (t * 128 >= n) return;  // past the end of a shorter sequence: nothing to do
  const int n_tiles_b = (n + 127) / 128;
  const int i0 = p.causal ? t : 0;
  const int n_q = n_tiles_b - i0;

  uint8_t* smem;
  uint32_t sbase, tmem;
  volatile int* abort_flag;
  if (!bwd_setup<L>(smem_raw, smem, sbase, p.epoch, abort_flag, tmem, warp)) return;
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};
  const int n_steps = p.group * n_q;
  auto step_head = [&](int s) { return b * p.Hq + hk * p.group + s / n_q; };  // b*Hq + h
  auto step_tile = [&](int s) { return i0 + s % n_q; };

  // A operand of the accumulator pre-load: ones in k = 0..2 of every row
  // (f16 1.0 = 0x3C00, bf16 1.0 = 0x3F80), same core-matrix layout as the
  // vector tiles; made visible to the tensor core's (async proxy) reads.
  if (threadIdx.x < 256) {
    const uint32_t one = BF16 ? 0x3F80u : 0x3C00u;
    const int row = threadIdx.x >> 1, half = threadIdx.x & 1;
    uint4* dst = reinterpret_cast<uint4*>(smem + L::kOffOnes + (row >> 3) * 256 + (row & 7) * 16 +
                                          half * 128);
    *dst = half ? make_uint4(0u, 0u, 0u, 0u) : make_uint4(one | (one << 16), one, 0u, 0u);
  }
  ptx::fence_proxy_async_smem();
  __syncthreads();

  if (warp == kBwdWarpLoad) {
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_last();
      ptx::mbar_arrive_expect_tx(bar(L::kBarFix), 2 * L::kTile);
#pragma unroll
      for (int c = 0; c < L::kColBlocks; ++c) {
        // fixed layout: (column, row, batch*head); packed: (column, head, row)
        const int c1 = p.cu ? hk : t * 128, c2 = p.cu ? start + t * 128 : bhk;
        ptx::tma_load_3d(sbase + L::kOffFix + c * L::kBlockBytes, &p.tm_k, bar(L::kBarFix), c * 64,
                         c1, c2, pol);
        ptx::tma_load_3d(sbase + L::kOffFix + L::kTile + c * L::kBlockBytes, &p.tm_v,
                         bar(L::kBarFix), c * 64, c1, c2, pol);
      }
      // ring item 2s: Q tile (+ its L2 vector), 2s+1: dO tile (+ its D vector)
      int issued = 0;
      for (int i = 0; i < 2 * n_steps; ++i) {
        const int slot = i % L::kSlots;
        if (i >= L::kSlots && !bar_wait(bar(L::kBarEmpty + slot), ((i / L::kSlots) - 1) & 1, wc, 41))
          break;
        const int s = i >> 1;
        if (!(i & 1)) FA_TRACE_AT(s, 16);
        const int bhq = step_head(s);
        const int qt = step_tile(s);
        const void* map = (i & 1) ? static_cast<const void*>(&p.tm_do) : static_cast<const void*>(&p.tm_q);
        const uint8_t* vec = p.vt + ((static_cast<size_t>(bhq) * p.n_tiles + qt) * 2 + (i & 1)) * L::kVec;
        ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile + L::kVec);
        const int c1 = p.cu ? bhq % p.Hq : qt * 128, c2 = p.cu ? start + qt * 128 : bhq;
#pragma unroll
        for (int c = 0; c < L::kColBlocks; ++c)
          ptx::tma_load_3d(sbase + L::kOffRing + slot * L::kTile + c * L::kBlockBytes, map,
                           bar(L::kBarFull + slot), c * 64, c1, c2, pol);
        ptx::bulk_load(sbase + L::kOffVec + slot * L::kVec, vec, L::kVec, bar(L::kBarFull + slot));
        issued = i + 1;
      }
      for (int i = max(0, issued - L::kSlots); i < issued; ++i)
        bar_wait(bar(L::kBarFull + i % L::kSlots), (i / L::kSlots) & 1, wc, 42, false);
      bar_wait(bar(L::kBarFix), 0, wc, 42, false);
    }
  } else if (warp == kBwdWarpMma) {
    // Issue order, step s (S^T and dP^T of step 0 first):
    //   [P^T(s) written]   dV += P^T(s) dO(s)   S^T(s+1)
    //   [dS^T(s) written]  dK += dS^T(s) Q(s)   dP^T(s+1)
    // The elementwise warps compute P^T(s) while dP^T(s) is still on the
    // tensor pipe and dS^T(s) while dV(s) and S^T(s+1) run.  S^T(s+1)
    // overwrites the TMEM columns of P^T(s) and dP^T(s+1) those of dS^T(s);
    // tcgen05.mma ops of one thread execute in issue order, so dV(s) / dK(s)
    // have read them first.
    constexpr uint32_t fmt = BF16 ? 1u : 0u;
    constexpr uint32_t idesc_s = ptx::make_idesc_f16(128, 128, fmt, 0, 0);
    constexpr uint32_t idesc_g = ptx::make_idesc_f16(128, D, fmt, 0, 1);
    auto slot_of = [](int i) { return i % L::kSlots; };
    auto phase_of = [](int i) { return static_cast<uint32_t>((i / L::kSlots) & 1); };
    auto wait = [&](uint32_t bb, uint32_t ph, int site) {
      return __all_sync(0xffffffffu, bar_wait_lean(bb, ph, wc, site));
    };
    const uint64_t k_desc = ptx::smem_desc_sw128(sbase + L::kOffFix, 16, 1024);
    const uint64_t v_desc = ptx::smem_desc_sw128(sbase + L::kOffFix + L::kTile, 16, 1024);
    const uint64_t ring_k = ptx::smem_desc_sw128(sbase + L::kOffRing, 16, 1024);              // K-major
    const uint64_t ring_mn = ptx::smem_desc_sw128(sbase + L::kOffRing, L::kBlockBytes, 1024);  // MN-major
    const uint64_t ones_desc = ptx::smem_desc_noswz(sbase + L::kOffOnes, 128, 256);
    // D = ones x vec^T + A B^T with A the fixed K (V) tile, B ring item `item`
    // (Q or dO, K = d) and vec the item's vector tile: the first product puts
    // -LSE/scale (-D) of each query column into every row of the accumulator
    auto issue_score = [&](uint32_t d_col, uint64_t a_desc, int item, uint32_t done_bar) {
      const uint64_t b_off = static_cast<uint64_t>((slot_of(item) * L::kTile) >> 4);
      const uint64_t vec_desc =
          ptx::smem_desc_noswz(sbase + L::kOffVec + slot_of(item) * L::kVec, 128, 256);
      if (ptx::elect_one()) {
        ptx::mma_ss(tmem + d_col, ones_desc, vec_desc, idesc_s, 0u);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
          ptx::mma_ss(tmem + d_col, a_desc + off, ring_k + b_off + off, idesc_s, 1u);
        }
        ptx::mma_commit(done_bar);
      }
      __syncwarp();
    };
    // acc += A B with A packed in TMEM (queries 64g.. of group g at columns
    // a_col + 64g ..+32) and B ring item `item` MN-major (K = the step's 128
    // queries, 16 rows = 2 KB per K step)
    auto issue_grad = [&](uint32_t acc_col, uint32_t a_col, int item, bool first) {
      const uint64_t b_off = static_cast<uint64_t>((slot_of(item) * L::kTile) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          ptx::mma_ts(tmem + acc_col, tmem + a_col + 8 * kk + (kk >= 4 ? 32 : 0),
                      ring_mn + b_off + static_cast<uint64_t>((kk * 2048) >> 4), idesc_g,
                      (!first || kk > 0) ? 1u : 0u);
      }
      __syncwarp();
    };
    bool ok = wait(bar(L::kBarFix), 0, 43);
    if (ok && n_steps > 0) {
      ok = wait(bar(L::kBarFull + slot_of(0)), phase_of(0), 44);
      if (ok) {
        ptx::tc_fence_after();
        issue_score(L::tS, k_desc, 0, bar(L::kBarS));
        ok = wait(bar(L::kBarFull + slot_of(1)), phase_of(1), 44);
      }
      if (ok) issue_score(L::tDP, v_desc, 1, bar(L::kBarS + 1));
    }
    for (int s = 0; ok && s < n_steps; ++s) {
      const bool next = s + 1 < n_steps;
      const int iq = 2 * s, id = 2 * s + 1;
      if (lane == 0) FA_TRACE_AT(s, 5);
      if (!(ok = wait(bar(L::kBarP), s & 1, 45))) break;
      if (lane == 0) FA_TRACE_AT(s, 1);
      ptx::tc_fence_after();
      issue_grad(L::tAcc0, L::tS, id, s == 0);  // dV += P^T dO
      if (next) {
        if (!(ok = wait(bar(L::kBarFull + slot_of(iq + 2)), phase_of(iq + 2), 44))) break;
        issue_score(L::tS, k_desc, iq + 2, bar(L::kBarS));  // S^T(s+1)
      }
      if (lane == 0) FA_TRACE_AT(s, 2);
      if (!(ok = wait(bar(L::kBarP + 1), s & 1, 45))) break;
      if (lane == 0) FA_TRACE_AT(s, 3);
      ptx::tc_fence_after();
      issue_grad(L::tAcc1, L::tDP, iq, s == 0);  // dK += dS^T Q
      // the step's Q / dO tiles and their vectors are read for the last time
      if (ptx::elect_one()) {
        ptx::mma_commit(bar(L::kBarEmpty + slot_of(iq)));
        ptx::mma_commit(bar(L::kBarEmpty + slot_of(id)));
      }
      __syncwarp();
      if (next) {
        if (!(ok = wait(bar(L::kBarFull + slot_of(id + 2)), phase_of(id + 2), 44))) break;
        issue_score(L::tDP, v_desc, id + 2, bar(L::kBarS + 1));  // dP^T(s+1)
      }
      if (lane == 0) FA_TRACE_AT(s, 4);
    }
    if (ptx::elect_one()) ptx::mma_commit(bar(L::kBarG));
    __syncwarp();
    bar_wait(bar(L::kBarG), 0, wc, 46, false);
    __syncwarp();
  } else if (warp < 8) {
    // rows = keys of tile t; group g takes queries [64g, 64g+64) of the step.
    // P^T stays in registers (fp32) between the two phases.
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int key = t * 128 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t col0 = 64u * g;
    const float sl = p.scale_log2;
    // padded batch: a key outside its entry's valid range gets P^T = 0;
    // packed: a row past the sequence's end (the next sequence's) too
    const bool key_ok = key < n && (p.k_lo == nullptr ||
                                    (key >= __ldg(p.k_lo + b) && key < __ldg(p.k_hi + b)));
    bool ok = true;
    for (int s = 0; ok && s < n_steps; ++s) {
      const int qt = step_tile(s);
      const bool diag = p.causal && qt == t;  // query < key is masked
      if (threadIdx.x == 0) FA_TRACE_AT(s, 8);
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS), s & 1, wc, 47));
      if (!ok) break;
      if (threadIdx.x == 0) FA_TRACE_AT(s, 9);
      ptx::tc_fence_after();
      float pr[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32];
        ptx::tmem_ld32(tmem + lane_off + L::tS + col0 + 32 * c, sv);
        ptx::tmem_wait_ld();
        pin_after_wait<32>(sv);
        if (threadIdx.x == 0) FA_TRACE_AT(s, c ? 15 : 13);
        // S^T already holds s - LSE/scale.  Diagonal tile: query
        // q = col0 + 32c + i is kept when q >= key r
        // (a key outside its range masks every column)
        if (diag || !key_ok)
          bwd_exp32<true>(pr + 32 * c, sv, sl, nullptr, 0.f,
                          key_ok ? r - static_cast<int>(col0) - 32 * c : 32, 32);
        else
          bwd_exp32<false>(pr + 32 * c, sv, sl, nullptr, 0.f, 0, 32);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack2<BF16>(pr[32 * c + 2 * i], pr[32 * c + 2 * i + 1]);
        if (threadIdx.x == 0) FA_TRACE_AT(s, c ? 17 : 14);
        // P^T into the group's S columns col0 + 16c.. (already read)
        ptx::tmem_st16(tmem + lane_off + L::tS + col0 + 16 * c, pk);
      }
      ptx::tmem_wait_st();
      if (threadIdx.x == 0) FA_TRACE_AT(s, 18);
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarP));
      if (threadIdx.x == 0) FA_TRACE_AT(s, 10);
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + 1), s & 1, wc, 47));
      if (!ok) break;
      if (threadIdx.x == 0) FA_TRACE_AT(s, 11);
      ptx::tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t dv[32];
        ptx::tmem_ld32(tmem + lane_off + L::tDP + col0 + 32 * c, dv);
        ptx::tmem_wait_ld();
        pin_after_wait<32>(dv);
        uint32_t gk[16];
        bwd_ds32<BF16, false>(gk, pr + 32 * c, dv, nullptr, 0.f);  // dP^T already holds dP - D
        // dS^T into the group's dP columns col0 + 16c.. (already read)
        ptx::tmem_st16(tmem + lane_off + L::tDP + col0 + 16 * c, gk);
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarP + 1));
      if (threadIdx.x == 0) FA_TRACE_AT(s, 12);
    }
    if (ok) ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarG), 0, wc, 48));
    if (ok) {
      // group 0 writes the dV rows, group 1 the dK rows
      ptx::tc_fence_after();
      const bool store = key < n;
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      // row index in units of d elements (packed: token-major [total, Hkv, d])
      const size_t row = p.cu ? static_cast<size_t>(start + key) * p.Hkv + hk
                              : static_cast<size_t>(bhk) * p.N + key;
      if (g == 0)
        bwd_store_row<D, BF16>(tmem + lane_off + L::tAcc0, 1.0f, reinterpret_cast<T*>(p.dv) + row * D, store);
      else
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
  // work: query tile t of (b, hq); key tiles 0..n_kv-1 (causal: j <= t,
  // heaviest tiles first within each group of kBwdHeadGroup heads)
  int t, bh;
  bwd_block_order(p.causal, static_cast<int>(blockIdx.x), p.B * p.Hq, p.n_tiles, t, bh);
  if (p.causal) t = p.n_tiles - 1 - t;
  const int b = bh / p.Hq;
  const int h = bh % p.Hq;
  const int bh_kv = b * p.Hkv + h / p.group;
  int start, n;  // sequence of batch entry b (packed varlen: its rows)
  bwd_seq(p.cu, p.total, p.N, b, start, n);
  if (t * 128 >= n) return;  // past the end of a shorter sequence: nothing to do
  const int n_kv = p.causal ? t + 1 : (n + 127) / 128;

  uint8_t* smem;
  uint32_t sbase, tmem;
  volatile int* abort_flag;
  if (!bwd_setup<L>(smem_raw, smem, sbase, p.epoch, abort_flag, tmem, warp)) return;
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};

  if (warp == kBwdWarpLoad) {
    if (lane == 0) {
      const uint64_t pol = ptx::policy_evict_last();
      ptx::mbar_arrive_expect_tx(bar(L::kBarFix), 2 * L::kTile);
#pragma unroll
      for (int c = 0; c < L::kColBlocks; ++c) {
        // fixed layout: (column, row, batch*head); packed: (column, head, row)
        const int c1 = p.cu ? h : t * 128, c2 = p.cu ? start + t * 128 : bh;
        ptx::tma_load_3d(sbase + L::kOffFix + c * L::kBlockBytes, &p.tm_q, bar(L::kBarFix), c * 64,
                         c1, c2, pol);
        ptx::tma_load_3d(sbase + L::kOffFix + L::kTile + c * L::kBlockBytes, &p.tm_do,
                         bar(L::kBarFix), c * 64, c1, c2, pol);
      }
      // ring item 2j: K_j, 2j+1: V_j
      int issued = 0;
      for (int i = 0; i < 2 * n_kv; ++i) {
        const int slot = i % L::kSlots;
        if (i >= L::kSlots && !bar_wait(bar(L::kBarEmpty + slot), ((i / L::kSlots) - 1) & 1, wc, 51))
          break;
        const void* map = (i & 1) ? static_cast<const void*>(&p.tm_v) : static_cast<const void*>(&p.tm_k);
        ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile);
        const int row = (i >> 1) * 128;
        const int c1 = p.cu ? h / p.group : row, c2 = p.cu ? start + row : bh_kv;
#pragma unroll
        for (int c = 0; c < L::kColBlocks; ++c)
          ptx::tma_load_3d(sbase + L::kOffRing + slot * L::kTile + c * L::kBlockBytes, map,
                           bar(L::kBarFull + slot), c * 64, c1, c2, pol);
        issued = i + 1;
      }
      for (int i = max(0, issued - L::kSlots); i < issued; ++i)
        bar_wait(bar(L::kBarFull + i % L::kSlots), (i / L::kSlots) & 1, wc, 52, false);
      bar_wait(bar(L::kBarFix), 0, wc, 52, false);
    }
  } else if (warp == kBwdWarpMma) {
    // Issue order, K/V tile j (S and dP of tile 0 first):
    //   [S(j) read]      S(j+1)
    //   [dS(j) written]  dQ += dS(j) K_j   dP(j+1)
    // dS has its own TMEM columns, so S(j+1) overwrites S(j) as soon as the
    // elementwise warps hold P(j) in registers; they compute P(j+1) while
    // dQ(j) and dP(j+1) run.  dP(j+1) overwrites dP(j) after they have read
    // it, and it completes after dQ(j) (issue order), before dS(j+1) is written.
    constexpr uint32_t fmt = BF16 ? 1u : 0u;
    constexpr uint32_t idesc_s = ptx::make_idesc_f16(128, 128, fmt, 0, 0);
    constexpr uint32_t idesc_g = ptx::make_idesc_f16(128, D, fmt, 0, 1);
    auto slot_of = [](int i) { return i % L::kSlots; };
    auto phase_of = [](int i) { return static_cast<uint32_t>((i / L::kSlots) & 1); };
    auto wait = [&](uint32_t bb, uint32_t ph, int site) {
      return __all_sync(0xffffffffu, bar_wait_lean(bb, ph, wc, site));
    };
    const uint64_t do_desc = ptx::smem_desc_sw128(sbase + L::kOffFix + L::kTile, 16, 1024);
    const uint64_t ring_k = ptx::smem_desc_sw128(sbase + L::kOffRing, 16, 1024);
    const uint64_t ring_mn = ptx::smem_desc_sw128(sbase + L::kOffRing, L::kBlockBytes, 1024);
    // D = A B^T with B ring item `item` (K or V), K = d, and A the fixed tile:
    // Q from TMEM (copied there by the elementwise warps; halves the product's
    // shared-memory reads) or dO from shared memory
    auto issue_score = [&](uint32_t d_col, bool a_in_tmem, int item, uint32_t done_bar) {
      const uint64_t b_off = static_cast<uint64_t>((slot_of(item) * L::kTile) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
          if (a_in_tmem)
            ptx::mma_ts(tmem + d_col, tmem + L::tQ + 8 * kk, ring_k + b_off + off, idesc_s,
                        kk > 0 ? 1u : 0u);
          else
            ptx::mma_ss(tmem + d_col, do_desc + off, ring_k + b_off + off, idesc_s, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(done_bar);
      }
      __syncwarp();
    };
    bool ok = wait(bar(L::kBarFix), 0, 53) && wait(bar(L::kBarQT), 0, 53);
    if (ok && n_kv > 0) {
      ok = wait(bar(L::kBarFull + slot_of(0)), phase_of(0), 54);
      if (ok) {
        ptx::tc_fence_after();
        issue_score(L::tS, true, 0, bar(L::kBarS));
        ok = wait(bar(L::kBarFull + slot_of(1)), phase_of(1), 54);
      }
      if (ok) issue_score(L::tDP, false, 1, bar(L::kBarS + 1));
    }
    for (int j = 0; ok && j < n_kv; ++j) {
      const bool next = j + 1 < n_kv;
      const int ik = 2 * j, iv = 2 * j + 1;
      if (lane == 0) FA_TRACE_AT(j, 19);
      if (!(ok = wait(bar(L::kBarP), j & 1, 55))) break;
      if (lane == 0) FA_TRACE_AT(j, 20);
      if (next) {
        if (!(ok = wait(bar(L::kBarFull + slot_of(ik + 2)), phase_of(ik + 2), 54))) break;
        ptx::tc_fence_after();
        issue_score(L::tS, true, ik + 2, bar(L::kBarS));  // S(j+1)
      }
      if (lane == 0) FA_TRACE_AT(j, 21);
      if (!(ok = wait(bar(L::kBarP + 1), j & 1, 55))) break;
      if (lane == 0) FA_TRACE_AT(j, 22);
      ptx::tc_fence_after();
      // dQ += dS K_j (A = dS from TMEM, B = K_j MN-major: K = keys)
      const uint64_t k_off = static_cast<uint64_t>((slot_of(ik) * L::kTile) >> 4);
      if (ptx::elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          ptx::mma_ts(tmem + L::tAcc0, tmem + L::tDS + 8 * kk,
                      ring_mn + k_off + static_cast<uint64_t>((kk * 2048) >> 4), idesc_g,
                      (j > 0 || kk > 0) ? 1u : 0u);
        ptx::mma_commit(bar(L::kBarEmpty + slot_of(ik)));  // K_j read
        ptx::mma_commit(bar(L::kBarEmpty + slot_of(iv)));  // V_j read
      }
      __syncwarp();
      if (next) {
        if (!(ok = wait(bar(L::kBarFull + slot_of(iv + 2)), phase_of(iv + 2), 54))) break;
        issue_score(L::tDP, false, iv + 2, bar(L::kBarS + 1));  // dP(j+1)
      }
      if (lane == 0) FA_TRACE_AT(j, 23);
    }
    if (ptx::elect_one()) ptx::mma_commit(bar(L::kBarG));
    __syncwarp();
    bar_wait(bar(L::kBarG), 0, wc, 56, false);
    __syncwarp();
  } else if (warp < 8) {
    // rows = queries of tile t; group g takes keys [64g, 64g+64) of each K/V tile
    const int g = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int q_row = t * 128 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int col0 = 64 * g;
    const float sl = p.scale_log2;
    const float nlv = p.l2[static_cast<size_t>(bh) * p.n_pad + q_row];  // -LSE*log2(e)
    const float ndv = p.dd[static_cast<size_t>(bh) * p.n_pad + q_row];  // -D
    const int k_begin = p.k_lo == nullptr ? 0 : __ldg(p.k_lo + b);
    const int k_end = p.k_lo == nullptr ? p.N : __ldg(p.k_hi + b);
    bool ok = true;
    if (g == 0) {
      // row r of the Q tile (TMA 128-byte swizzle: 16-byte chunk c of a row
      // at position c ^ (r % 8)) into TMEM lane r, element pairs packed per
      // column: the A operand layout of the TS product S = Q K^T
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarFix), 0, wc, 59));
      if (ok) {
#pragma unroll
        for (int blk = 0; blk < L::kColBlocks; ++blk) {
          uint32_t w[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = *reinterpret_cast<const uint4*>(
                smem + L::kOffFix + blk * L::kBlockBytes + r * 128 + ((c ^ (r & 7)) * 16));
            w[4 * c] = v.x;
            w[4 * c + 1] = v.y;
            w[4 * c + 2] = v.z;
            w[4 * c + 3] = v.w;
          }
          ptx::tmem_st32(tmem + lane_off + L::tQ + 32 * blk, w);
        }
        ptx::tmem_wait_st();
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarQT));
    }
    for (int j = 0; ok && j < n_kv; ++j) {
      // keys >= N, (causal) keys > this query and (padded batch) keys outside
      // the entry's range get P = 0; [klo, lim) relative to the group's first key
      const int key0 = j * 128 + col0;
      int lim = n - key0;
      if (p.causal && j == t) lim = min(lim, r + 1 - col0);
      int klo = 0;
      if (p.k_lo != nullptr) {
        klo = k_begin - key0;
        lim = min(lim, k_end - key0);
      }
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS), j & 1, wc, 57));
      if (!ok) break;
      if (threadIdx.x == 0) FA_TRACE_AT(j, 25);
      ptx::tc_fence_after();
      // masked tiles only: the group's keys reach N, the diagonal or a range end
      const bool masked = (p.causal && j == t) || n - key0 < 64 || klo > 0 ||
                          (p.k_lo != nullptr && k_end - key0 < 64);
      if (threadIdx.x == 0) FA_TRACE_AT(j, 24);
      float pr[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32];
        ptx::tmem_ld32(tmem + lane_off + L::tS + col0 + 32 * c, sv);
        ptx::tmem_wait_ld();
        pin_after_wait<32>(sv);
        if (masked)
          bwd_exp32<true>(pr + 32 * c, sv, sl, nullptr, nlv, klo - 32 * c, lim - 32 * c);
        else
          bwd_exp32<false>(pr + 32 * c, sv, sl, nullptr, nlv, 0, 32);
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarP));  // S(j) read: S(j+1) may overwrite it
      if (threadIdx.x == 0) FA_TRACE_AT(j, 26);
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + 1), j & 1, wc, 57));
      if (!ok) break;
      if (threadIdx.x == 0) FA_TRACE_AT(j, 27);
      ptx::tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t dv[32];
        ptx::tmem_ld32(tmem + lane_off + L::tDP + col0 + 32 * c, dv);
        ptx::tmem_wait_ld();
        pin_after_wait<32>(dv);
        uint32_t gk[16];
        bwd_ds32<BF16, true>(gk, pr + 32 * c, dv, nullptr, ndv);
        ptx::tmem_st16(tmem + lane_off + L::tDS + 32 * g + 16 * c, gk);
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar(L::kBarP + 1));  // dS(j) written
      if (threadIdx.x == 0) FA_TRACE_AT(j, 28);
    }
    if (ok) ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarG), 0, wc, 58));
    if (ok && g == 0) {
      ptx::tc_fence_after();
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      // row index in units of d elements (packed: token-major [total, Hq, d])
      const size_t row = p.cu ? static_cast<size_t>(start + q_row) * p.Hq + h
                              : static_cast<size_t>(bh) * p.N + q_row;
      // rows that take no part (padding, or no visible key: -LSE = -inf) get dQ = 0
      bwd_store_row<D, BF16>(tmem + lane_off + L::tAcc0, nlv == -INFINITY ? 0.f : p.scale,
                             reinterpret_cast<T*>(p.dq) + row * D, q_row < n);
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
  const long long rows_per_block = 256 / (D / 8);
  fa_bwd_prep_kernel<BF16><<<static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block), 256, 0, stream>>>(
      o, dout, lse, const_cast<float*>(p.l2), const_cast<float*>(p.dd), const_cast<uint8_t*>(p.vt),
      p.scale, p.N, p.n_pad, rows, D, p.Hq, p.q_lo, p.q_hi, p.cu, p.total);
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
