// FlashAttention forward for B200 (sm_100a).
//
//   O = softmax(Q K^T * scale) V      (+ LSE = logsumexp(Q K^T * scale) per row)
//
// Replaces the sm_75 WMMA kernels of the reference
// (src/kernels/flash_attention_forward.cu:345-791,
//  flash-attention-sm75-fused/src/flash_mha_flatargs.cu:86-226,
//  flash-attention-sm75-fused/src/flash_mha_v2.cu:165-361) with one
// warp-specialised tcgen05 kernel.  The math is the same online softmax
// (flash-attention-sm75-fused/include/online_step.cuh:36-126): running row
// max m, running sum l, O rescaled by exp(m_old - m_new), O / l at the end.
//
// One CTA owns a "Q pair": two 128-row tiles of one (batch, query-head).
//   warps 0-3  softmax group 0  (rows   0..127 of the pair, one row / thread)
//   warps 4-7  softmax group 1  (rows 128..255)
//   warp  8    TMA producer     (Q once, K/V tiles through a ring of slots)
//   warp  9    MMA issuer       (tcgen05.mma from one elected lane) + TMEM owner
//   warps 10-11 idle (complete the producer warpgroup for setmaxnreg)
//
// Tensor memory (512 columns x 128 lanes, lane = query row of a tile):
//   S_g  = Q_g K_j^T        fp32, 128 columns per group
//   P_g  = exp2(S_g - m)    f16/bf16 pairs, 64 columns (aliases S_g when d=128)
//   O_g += P_g V_j          fp32, d columns per group
// QK^T reads both operands from shared memory; PV reads P from TMEM.
//
// Causal masking is top-left aligned (key j visible to query i iff j <= i),
// as in src/reference/attention_ref.py:33-40.  Tiles above the diagonal are
// never loaded or multiplied; the diagonal tile is masked in registers.
// GQA maps query head h to KV head h / (Hq/Hkv), the mapping that
// repeat_interleave gives in src/flash_attention_sm75/ops.py:24-26, without
// materialising the repeated K/V.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "fa_fwd.h"
#include "sm100_ptx.cuh"
#include "fa_softmax.cuh"

namespace fa {

// Sticky device status: high 32 bits = launch epoch, low 32 bits = error code.
// Written only when a bounded wait expires; read by fa_device_status().
__device__ unsigned long long g_fa_status = 0ull;

// Work-item counters of persistent launches whose last rounds are dealt
// dynamically: slot sched % kSchedSlots holds (sched << 32) | items handed
// out.  A launch starts its slot by replacing a value tagged with another
// launch's number, so no reset is needed between launches; 256 slots keep
// launches whose CTAs run at the same time apart (the host numbers these
// launches on their own counter).
constexpr unsigned kSchedSlots = 256;
__device__ unsigned long long g_fa_sched[kSchedSlots];

namespace {

constexpr int kBlockM = 128;  // query rows per tile (one TMEM lane each)
constexpr int kBlockN = 128;  // keys per K/V tile
constexpr int kThreads = 384;   // 3 warpgroups
// Warpgroup of the producer, the MMA issuer and two spare warps (8-11); the
// two softmax warpgroups are warps 0-7.
constexpr int kWarpLoad = 8;
constexpr int kWarpMma = 9;
constexpr int kWarpSoftmax0 = 0;
// Register split: launched at kLaunchRegs per thread (65536 / 384 rounded down
// to a multiple of 8); the producer/MMA warpgroup gives registers to the two
// softmax warpgroups.  256*kRegsSoftmax + 128*kRegsOther must not exceed
// 384*kLaunchRegs.
constexpr int kLaunchRegs = 168;
constexpr int kRegsSoftmax = 192;
constexpr int kRegsOther = 120;
static_assert(256 * kRegsSoftmax + 128 * kRegsOther <= kThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
// Lazy rescaling: O and l keep a stale row max until the true max exceeds it
// by more than 2^15 (log2 units), so P = exp2(s - m_stale) <= 2^15 still fits
// f16 (max 65504) and bf16; results are identical up to rounding.
constexpr float kRescaleThreshold = 15.0f;

template <int D>
struct Layout {
  static constexpr int kColBlocks = D / 64;       // 128-byte swizzle column blocks
  static constexpr int kBlockBytes = kBlockM * 128;  // one 64-column block of a 128-row tile
  static constexpr int kTile = kBlockM * D * 2;   // bytes of a 128-row f16 tile
  // K and V tiles stream through one ring of tile-sized slots in load order
  // K0 V0 K1 V1 ...; a slot is refilled once the MMAs reading it completed.
  static constexpr int kSlots = (D == 128) ? 5 : 8;
  // shared memory (offsets from a 1024-aligned base)
  static constexpr int kOffQ = 0;                 // Q0, Q1
  static constexpr int kOffKV = 2 * kTile;        // ring slot s at kOffKV + s*kTile
  static constexpr int kOffBar = kOffKV + kSlots * kTile;
  // barrier indices
  static constexpr int kBarQ = 0;                       // 2
  static constexpr int kBarFull = 2;                    // kSlots (TMA tx-count)
  static constexpr int kBarEmpty = kBarFull + kSlots;   // kSlots (MMA commit)
  static constexpr int kBarS = kBarEmpty + kSlots;      // 2
  static constexpr int kBarP = kBarS + 2;               // 2
  static constexpr int kBarO = kBarP + 2;               // 2
  static constexpr int kBarDrain = kBarO + 2;           // 1
  // persistent launches (several work items per CTA): the MMAs that read Q
  // buffer b for one item have completed, so the next Q may overwrite it
  static constexpr int kBarQFree = kBarDrain + 1;       // 2
  // early part of P_g written (kPEarlyQuarters x 32 keys): the PV MMA starts
  // on it while the softmax computes the rest (128 arrivals)
  static constexpr int kBarPH = kBarQFree + 2;          // 2
  // dynamically dealt rounds: the producer publishes each round's work item
  // in a 4-entry queue (full: producer arrival; empty: every softmax thread
  // and lane 0 of the MMA warp have read it)
  static constexpr int kItemQ = 4;
  static constexpr int kBarItemFull = kBarPH + 2;               // kItemQ
  static constexpr int kBarItemEmpty = kBarItemFull + kItemQ;   // kItemQ
  static constexpr int kNumBars = kBarItemEmpty + kItemQ;
  static constexpr int kOffMisc = kOffBar + 8 * kNumBars;
  static constexpr int kOffItemQ = kOffMisc + 16;               // kItemQ ints
  // dual-tile items (d = 64): each softmax thread's (m, l) for the in-CTA
  // merge of the two groups' key halves, double-buffered by work item
  static constexpr int kOffXchg = kOffItemQ + 4 * kItemQ;
  static constexpr int kXchgBytes = (D == 64) ? 2 * 2 * kBlockM * 8 : 0;
  static constexpr int kBytes = kOffXchg + kXchgBytes;
  static constexpr int kDynBytes = kBytes + 1024;  // slack for 1024-byte alignment
  // tensor memory columns
  static constexpr uint32_t kTmemCols = 512;
  __host__ __device__ static constexpr uint32_t tS(int g) { return g ? 128u : 0u; }
  __host__ __device__ static constexpr uint32_t tO(int g) { return g ? 256u + D : 256u; }
  // d=128 fills TMEM, so P overwrites the S columns it was computed from;
  // d=64 leaves room for separate P columns.
  static constexpr bool kAliasP = (D == 128);
  __host__ __device__ static constexpr uint32_t tP(int g) {
    return kAliasP ? tS(g) : (g ? 448u : 384u);
  }
  static_assert(kDynBytes <= 227 * 1024, "shared memory budget");
};

constexpr uint32_t kSuspendNs = 100000;  // upper bound of one hardware-suspended wait

struct WaitCtl {
  volatile int* abort;        // CTA-wide abort flag in shared memory
  unsigned long long timeout_ns;
  unsigned epoch;
};

__device__ void record_error(unsigned epoch, int code) {
  const unsigned long long want =
      (static_cast<unsigned long long>(epoch) << 32) | static_cast<unsigned>(code);
  unsigned long long old = atomicAdd(&g_fa_status, 0ull);
  while (true) {
    if ((old >> 32) == epoch && (old & 0xffffffffull) != 0ull) return;  // first error wins
    const unsigned long long prev = atomicCAS(&g_fa_status, old, want);
    if (prev == old) return;
    old = prev;
  }
}

// Next work-item number of launch `sched` from its counter slot (0, 1, 2, ...
// in the order of the calls across the launch's CTAs), or -1 (error recorded,
// CTA aborting) if the counter could not be updated after many attempts.
__device__ int sched_take(unsigned sched, const WaitCtl& c) {
  unsigned long long* ctr = &g_fa_sched[sched % kSchedSlots];
  unsigned long long v = atomicAdd(ctr, 0ull);
  for (int i = 0; i < (1 << 20); ++i) {
    const bool mine = static_cast<unsigned>(v >> 32) == sched;
    const unsigned long long nv =
        mine ? v + 1ull : ((static_cast<unsigned long long>(sched) << 32) | 1ull);
    const unsigned long long prev = atomicCAS(ctr, v, nv);
    if (prev == v) return mine ? static_cast<int>(v & 0xffffffffull) : 0;
    v = prev;
  }
  *c.abort = 1;
  record_error(c.epoch, FA_ERR_TIMEOUT_BASE + 6);
  return -1;
}

__device__ __forceinline__ bool bar_wait_slow(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                           int site, bool respect_abort) {
  const uint64_t t0 = ptx::global_timer_ns();
  while (true) {
    // sleeps in hardware until the phase completes or ~kSuspendNs elapse
    if (ptx::mbar_try_wait_sleep(bar, parity, kSuspendNs)) return true;
    if (respect_abort && *c.abort) return false;
    if (ptx::global_timer_ns() - t0 > c.timeout_ns) {
      *c.abort = 1;
      record_error(c.epoch, FA_ERR_TIMEOUT_BASE + site);
      return false;
    }
  }
}

// Bounded mbarrier wait.  Returns false if the CTA is aborting or the wait
// exceeded the watchdog deadline (which also records the error and aborts).
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, const WaitCtl& c, int site,
                                         bool respect_abort = true) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return bar_wait_slow(bar, parity, c, site, respect_abort);
}

// The slow path as a call, for warps with registers to spare: their code
// stays compact around every wait.
__device__ __noinline__ bool bar_wait_slow_call(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                                int site, bool respect_abort) {
  return bar_wait_slow(bar, parity, c, site, respect_abort);
}
__device__ __forceinline__ bool bar_wait_lean(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                              int site, bool respect_abort = true) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return bar_wait_slow_call(bar, parity, c, site, respect_abort);
}

// Bounded wait that polls without suspending the thread: for short waits on
// the critical path, where a suspended thread may resume late.  The timer is
// read every 256 polls.
__device__ __noinline__ bool bar_wait_spin_slow(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                                int site) {
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (ptx::mbar_test_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (*c.abort) return false;
      if (ptx::global_timer_ns() - t0 > c.timeout_ns) {
        *c.abort = 1;
        record_error(c.epoch, FA_ERR_TIMEOUT_BASE + site);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool bar_wait_spin(uint32_t bar, uint32_t parity, const WaitCtl& c,
                                              int site) {
  if (ptx::mbar_test_wait(bar, parity)) return true;
  return bar_wait_spin_slow(bar, parity, c, site);
}

// Make the values produced by tcgen05.ld visible to ordinary instructions
// only after tcgen05.wait::ld (the empty volatile asm cannot move above it).
template <int N>
__device__ __forceinline__ void pin_after_wait(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// Timeline tracing for development builds (-DFA_TRACE): the first
// kTraceCtas CTAs record clock64() at fixed points of every K/V tile into
// p.trace[cta][tile][event].  Compiled out otherwise.  Events of tile j:
//   0-3   MMA warp starts issuing PV0(j), S0(j+1), PV1(j), S1(j+1)
//   4, 5  MMA warp has issued PV0(j), S0(j+1)
//   6, 7  MMA warp before / after the V_j and K_{j+1} waits
//   8-15  softmax warp w arrived on P (w = 0..7)
//   16-23 softmax warp w saw S complete
//   24-27 observer warps (d=128): S0(j), PV0(j), S1(j), PV1(j) complete
//   28-29 group 0 / 1 tile max computed (row 0)
//   30-31 producer issued the loads of V_j / K_{j+1}
//   (tile kTraceTiles-1, events 30 / 31: CTA set up / CTA done)
// Dual (decode) launches index rows by each group's running tile count
// (mod 64) and record: 2g MMA warp saw V_j, K_{j+1} of group g land; 4+g
// P_g(j) seen and PV issued; 1+2g S_g(j+1) issued; 24+g / 26+g producer
// issued K / V of the tile; 8-23, 28-29 as above.
constexpr int kTraceCtas = 8, kTraceTiles = 64, kTraceEvents = 32;
#ifdef FA_TRACE
#define FA_TRACE_AT(tile, ev)                                                          \
  do {                                                                                 \
    if (p.trace != nullptr && blockIdx.x < kTraceCtas && (tile) < kTraceTiles)         \
      p.trace[(blockIdx.x * kTraceTiles + (tile)) * kTraceEvents + (ev)] = clock64(); \
  } while (0)
#else
#define FA_TRACE_AT(tile, ev) \
  do {                        \
  } while (0)
#endif

// The first kPEarlyQuarters quarters of P (32 keys each) are announced to the
// MMA warp before the rest is computed, so the PV steps on them overlap the
// softmax's tail.
#ifndef FA_P_EARLY_QUARTERS
#define FA_P_EARLY_QUARTERS 2
#endif
constexpr int kPEarlyQuarters = FA_P_EARLY_QUARTERS;
static_assert(kPEarlyQuarters >= 1 && kPEarlyQuarters <= 3, "early part of P: 1-3 quarters");

// exp2(x * sl - m) for the 128 scores of this thread's row; the packed
// f16/bf16 values go to TMEM (P operand of the PV MMA) in four 16-column
// quarters, the first kPEarlyQuarters announced (`announce()`, an mbarrier
// arrival) as soon as they are written; returns their fp32 sum.
template <bool BF16, bool kEmulate, int kPeriod = kEmuPeriod, typename Announce>
__device__ __forceinline__ float exp_tile(const float (&x)[kBlockN], float sl, float neg_m,
                                          uint32_t tP, Announce announce) {
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const int i = 32 * h + 2 * c;
      float e0, e1;
      exp2_pair<kEmulate, kPeriod>(c, x[i], x[i + 1], sl, neg_m, e0, e1);
      if (c & 1)
        ptx::fadd2(b0, b1, b0, b1, e0, e1);
      else
        ptx::fadd2(a0, a1, a0, a1, e0, e1);
      pk[c] = pack2<BF16>(e0, e1);
    }
    ptx::tmem_st16(tP + 16 * h, pk);
    if (h == kPEarlyQuarters - 1) {
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      announce();
    }
  }
  ptx::fadd2(a0, a1, a0, a1, b0, b1);
  return a0 + a1;
}

// Period of the pair kernel's exponential emulation pattern (one pair in
// kPairEmuPeriod on the polynomial): 1 in 8 at d = 128, 1 in 4 at d = 64.
// Measured on B200, interleaved runs: 1 in 8 against 1 in 4 gave C5 +2.5 %,
// C4 +0.6 %, C3 (d = 64) -1.7 %; 3 in 8 and 1 in 2 were slower everywhere
// (C5 -2 % / -11 %, C3 -7 % / -16 %): every polynomial adds softmax
// instructions that compete with the MMA warp for issue slots.
#ifndef FA_EMU_PERIOD_D128
#define FA_EMU_PERIOD_D128 8
#endif
template <int D>
constexpr int kPairEmuPeriod = (D == 128) ? FA_EMU_PERIOD_D128 : kEmuPeriod;

// One unit of work of a CTA: a (batch*head, Q pair, key split) triple, with
// the K/V tiles each softmax group processes.  A launch has n_work of them;
// CTA c takes c, c + gridDim.x, ... (one each unless the launch is persistent).
struct WorkItem {
  int bh, qp, sp, bh_kv, q_row0;
  bool has_q1;
  int n_kv[2];  // K/V tiles of group g (0: the group idles in this item)
  int jb[2];    // first K/V tile of group g
  int n_loop;   // max(n_kv)
  int n_items;  // K/V ring items the item loads
  // The item's sequence: nq query rows and nk keys (local row r, key j).
  int nq, nk;
  int causal_off;      // key j visible to local row r iff j <= r % pos_mod + causal_off
  int qy, qz, ky, kz;  // TMA row base and plane (head) of Q and K/V
};

// O element offset (rows o_rs apart) and LSE index (rows 1 apart) of local
// query row 0 of work item w, and its number of query rows.  Recomputed for
// the epilogue rather than kept live through the softmax loop.
// Work item (without its split) -> (Q pair from the heavy end, batch*head).
// Non-causal: head-major.  Causal pairs differ in work: items go pair-major
// within groups of p.head_group heads and head-major across groups, so each
// group starts its heaviest pairs first while the CTAs that run together
// still share a few heads' K/V in L2 (the host picks the group size:
// kFwdHeadGroup, or all heads for launches of at most two waves).
__device__ __forceinline__ void item_order(const FwdParams& p, int rest, int& qp_heavy, int& bh) {
  if (!p.causal) {
    qp_heavy = rest % p.n_qpairs;
    bh = rest / p.n_qpairs;
    return;
  }
  const int n_heads = p.B * p.heads;
  const int hg = max(p.head_group, 1);
  const int per_group = hg * p.n_qpairs;
  const int g = rest / per_group;
  const int r = rest % per_group;
  const int g_heads = min(hg, n_heads - g * hg);
  qp_heavy = r / g_heads;
  bh = g * hg + r % g_heads;
}

__device__ __forceinline__ void item_out(const FwdParams& p, int w, long long& o_row0,
                                         long long& lse_row0, int& nq) {
  int qp_unused, bh;
  item_order(p, w / p.n_splits, qp_unused, bh);
  if (p.ranges == 0) {
    nq = p.Nq;
    lse_row0 = static_cast<long long>(bh) * p.Nq;
    o_row0 = lse_row0 * p.o_rs;
    return;
  }
  const int b = bh / p.heads;
  const int ql = min(max(__ldg(p.q_lo + b), 0), p.q_lim);
  nq = min(max(__ldg(p.q_hi + b), ql), p.q_lim) - ql;
  if (p.ranges == 1) {
    const int hq = bh % p.heads;
    o_row0 = static_cast<long long>(ql) * p.o_rs + static_cast<long long>(hq) * (p.o_rs / p.heads);
    lse_row0 = static_cast<long long>(hq) * p.q_lim + ql;
  } else {
    lse_row0 = static_cast<long long>(bh) * p.Nq + ql;
    o_row0 = lse_row0 * p.o_rs;
  }
}

__device__ __forceinline__ void decode_item(const FwdParams& p, int w, WorkItem& it) {
  it.sp = w % p.n_splits;
  int qp;
  item_order(p, w / p.n_splits, qp, it.bh);
  if (p.causal) qp = p.n_qpairs - 1 - qp;  // causal: heaviest pairs first
  it.qp = qp;
  const int b = it.bh / p.heads;
  const int hq = it.bh % p.heads;
  it.bh_kv = b * p.Hkv + hq / p.group;
  // dual-tile items (dual == 2) are one 128-row Q tile each
  it.q_row0 = p.dual == 2 ? qp * kBlockM : qp * 2 * kBlockM;
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
    if (p.ranges == 1) {  // packed varlen: planes are heads, rows are tokens
      it.causal_off = p.causal_off + (p.causal_br ? it.nk - it.nq : 0);
      it.qz = hq;
      it.kz = hq / p.group;
    } else {  // padded batch: the absolute causal rule in local rows
      it.causal_off = p.causal_off + ql - kl;
      it.qz = it.bh;
      it.kz = it.bh_kv;
    }
    n_kv_tiles = (it.nk + kBlockN - 1) / kBlockN;
  }
  it.has_q1 = it.q_row0 + kBlockM < it.nq;
  auto tiles_of = [&](int t) {
    return kv_tiles_core(p.causal, it.nq, n_kv_tiles, it.causal_off, p.pos_mod, t);
  };
  const int j_begin = it.sp * p.tiles_per_split;
  if (p.dual) {
    // both groups on the item's Q tile; the split's tiles are halved
    // between them
    const int n = max(0, min(tiles_of(p.dual == 2 ? qp : 2 * qp), j_begin + p.tiles_per_split) -
                             j_begin);
    it.n_kv[0] = (n + 1) / 2;
    it.n_kv[1] = n / 2;
    it.jb[0] = j_begin;
    it.jb[1] = j_begin + it.n_kv[0];
  } else {
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      const int total = (g == 0 || it.has_q1) ? tiles_of(2 * qp + g) : 0;
      it.n_kv[g] = max(0, min(total, j_begin + p.tiles_per_split) - j_begin);
      it.jb[g] = j_begin;
    }
  }
  it.n_loop = max(it.n_kv[0], it.n_kv[1]);
  it.n_items = p.dual ? 2 * (it.n_kv[0] + it.n_kv[1]) : 2 * it.n_loop;
}

// Item index (load order, from 0 within the work item) of group g's K tile of
// iteration i; its V tile is the next item.  Shared mode: one K/V pair per
// iteration read by both groups.  Dual mode: K0 V0 K1 V1 per iteration while
// both groups have tiles (n_kv[0] >= n_kv[1]), then K0 V0.
__device__ __forceinline__ int k_item_of(const WorkItem& it, bool dual, int g, int i) {
  if (!dual) return 2 * i;
  return i < it.n_kv[1] ? 4 * i + 2 * g : 2 * it.n_kv[1] + 2 * i;
}

// Inverse of k_item_of: K/V tile of item index i (g = its group).
__device__ __forceinline__ int tile_of_item(const WorkItem& it, bool dual, int i, int& g) {
  int iter;
  if (!dual) {
    iter = i >> 1;
    g = 0;
  } else if (i < 4 * it.n_kv[1]) {
    iter = i >> 2;
    g = (i >> 1) & 1;
  } else {
    iter = it.n_kv[1] + ((i - 4 * it.n_kv[1]) >> 1);
    g = 0;
  }
  return (g ? it.jb[1] : it.jb[0]) + iter;
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1) fa_fwd_kernel(const __grid_constant__ FwdParams p) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kOffBar + 8u * static_cast<uint32_t>(i); };

  const bool dual = p.dual != 0;
  const int n_all = p.n_qpairs * p.B * p.heads * p.n_splits;
  const int n_work = p.item_end > 0 ? min(p.item_end, n_all) : n_all;
  const int w0 = p.item0 + static_cast<int>(blockIdx.x);
  // Work item of this CTA's k-th round.  Persistent launches outside dual
  // mode deal the rounds out boustrophedon-wise (odd rounds in reverse CTA
  // order), so CTAs that got the heavier item of one round get a lighter
  // one in the next (causal items are ordered heaviest first).
  const bool snake = !dual && p.n_ctas > 0;
  auto work_of = [&](int round) {
    const int c = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
    return p.item0 + round * G + ((snake && (round & 1)) ? (G - 1 - c) : c);
  };

  // ---- set-up: skip the CTA if this launch already failed elsewhere
  if (threadIdx.x == 0) {
    const unsigned long long st = *reinterpret_cast<volatile unsigned long long*>(&g_fa_status);
    *abort_flag = ((st >> 32) == p.epoch && (st & 0xffffffffull) != 0ull) ? 1 : 0;
    for (int i = 0; i < L::kNumBars; ++i) {
      // P completes on an arrival of every thread of a softmax group
      const bool is_p = (i == L::kBarP || i == L::kBarP + 1 || i == L::kBarPH ||
                         i == L::kBarPH + 1);
      const bool is_item_empty = i >= L::kBarItemEmpty && i < L::kBarItemEmpty + L::kItemQ;
      ptx::mbar_init(bar(i), is_p ? 128u : is_item_empty ? 257u : 1u);
    }
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (*abort_flag) return;
  if (warp == kWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), L::kTmemCols);
    ptx::tmem_relinquish();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const WaitCtl wc{abort_flag, p.timeout_ns, p.epoch};
  if (threadIdx.x == 0) FA_TRACE_AT(kTraceTiles - 1, 30);  // CTA set up

  // Rounds >= p.sched_round of a persistent shared-mode launch with
  // p.sched != 0 are dealt dynamically: this CTA's producer takes the next
  // number n from the launch's counter (item item0 + sched_round * G + n)
  // when it moves on, and publishes it in a shared 4-entry queue that the
  // MMA warp and the softmax groups read; a number >= n_work (the items ran
  // out) ends every role's loop.  Round r uses queue entry
  // (r - sched_round) % kItemQ.  Earlier rounds keep the static deal: CTAs
  // that run their rounds in step read the same heads' K/V at the same time
  // (measured: dealing every round dynamically balanced C5 causal perfectly
  // but ran 8 % slower, 2 % of it the queue hand-offs).
  const bool dyn = snake && p.sched != 0u;
  volatile int* item_q = reinterpret_cast<volatile int*>(smem + L::kOffItemQ);
  auto produce_item = [&](int round, bool& ok) -> int {
    if (!dyn || round < p.sched_round) return work_of(round);
    if (!ok) return n_work;
    const int q = round - p.sched_round, qs = q % L::kItemQ;
    if (q >= L::kItemQ &&
        !(ok = bar_wait(bar(L::kBarItemEmpty + qs), ((q / L::kItemQ) - 1) & 1, wc, 4)))
      return n_work;
    const int n = sched_take(p.sched, wc);
    if (n < 0) ok = false;
    const int w = n < 0 ? n_work : p.item0 + p.sched_round * static_cast<int>(gridDim.x) + n;
    item_q[qs] = w;
    ptx::mbar_arrive(bar(L::kBarItemFull + qs));  // release: the entry is visible to waiters
    return w;
  };
  // Every thread of the calling warp waits and reads; threads with `arrive`
  // (each softmax thread, lane 0 of the MMA warp: 257 arrivals) release it.
  auto consume_item = [&](int round, bool& ok, bool arrive) -> int {
    if (!dyn || round < p.sched_round) return work_of(round);
    if (!ok) return n_work;
    const int q = round - p.sched_round, qs = q % L::kItemQ;
    if (!(ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarItemFull + qs), (q / L::kItemQ) & 1,
                                                wc, 5))))
      return n_work;
    const int w = item_q[qs];
    if (arrive) ptx::mbar_arrive(bar(L::kBarItemEmpty + qs));
    return w;
  };

  if (warp < kWarpSoftmax0 || warp >= kWarpSoftmax0 + 8) {
   // ------------------------------------------------ producer warpgroup
   ptx::setmaxnreg_dec<kRegsOther>();
   if (warp == kWarpLoad) {
    // ===================================================== TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&p.tm_q);
      ptx::prefetch_tmap(&p.tm_k);
      ptx::prefetch_tmap(&p.tm_v);
      const uint64_t pol_q = ptx::policy_evict_first();
      const uint64_t pol_kv = ptx::policy_evict_last();
      const bool skip_q = (p.debug_flags & FA_DEBUG_SKIP_Q_LOAD) != 0;
      // Ring items are numbered across the CTA's work items (slot r % kSlots),
      // so the next item's K/V tiles load while the current one computes.
      // Dual mode double-buffers Q (work item k uses buffer k & 1): loading
      // item k's Q waits until the MMAs of item k-2, which read that buffer,
      // have completed.  Shared mode uses Q buffer g for group g's tile; a
      // persistent launch refills it after the previous item's last S_g.
      int ring = 0, k = 0, q_loads[2] = {0, 0};
#ifdef FA_TRACE
      int pc[2] = {0, 0};  // dual mode: tiles of group g in earlier work items (trace rows)
#endif
      bool ok = true;
      for (int w = w0; ok && w < n_work; w = produce_item(++k, ok)) {
        WorkItem it;
        decode_item(p, w, it);
        if (!skip_q) {
          if (dual) {
            const int qb = k & 1;
            if (k >= 2 && !(ok = bar_wait(bar(L::kBarQFree + qb), ((k - 2) >> 1) & 1, wc, 3)))
              break;
            ptx::mbar_arrive_expect_tx(bar(L::kBarQ + qb), L::kTile);
#pragma unroll
            for (int c = 0; c < L::kColBlocks; ++c)
              ptx::tma_load_3d(sbase + L::kOffQ + qb * L::kTile + c * L::kBlockBytes, &p.tm_q,
                               bar(L::kBarQ + qb), c * 64, it.qy + it.q_row0, it.qz, pol_q);
            if (qb) ++q_loads[1]; else ++q_loads[0];
          } else {
            // a group without K/V tiles needs no Q (the MMA warp waits for
            // Q tile g only when n_kv[g] > 0).  Persistent launches: Q buffer
            // g is refilled once the previous item's last S_g has completed.
            for (int g = 0; g < 2 && ok; ++g) {
              if (it.n_kv[g] == 0) continue;
              if (q_loads[g] > 0 &&
                  !(ok = bar_wait(bar(L::kBarQFree + g), (q_loads[g] - 1) & 1, wc, 3)))
                break;
              ptx::mbar_arrive_expect_tx(bar(L::kBarQ + g), L::kTile);
              const int row = it.qy + it.q_row0 + g * kBlockM;
#pragma unroll
              for (int c = 0; c < L::kColBlocks; ++c) {
                const int c0 = c * 64;
                if (p.ranges == 1)
                  ptx::tma_load_3d(sbase + L::kOffQ + g * L::kTile + c * L::kBlockBytes, &p.tm_q,
                                   bar(L::kBarQ + g), c0, it.qz, row, pol_q);
                else
                  ptx::tma_load_3d(sbase + L::kOffQ + g * L::kTile + c * L::kBlockBytes, &p.tm_q,
                                   bar(L::kBarQ + g), c0, row, it.qz, pol_q);
              }
              ++q_loads[g];
            }
            if (!ok) break;
          }
        }
        for (int i = 0; i < it.n_items; ++i, ++ring) {
          const int slot = ring % L::kSlots;
          if (ring >= L::kSlots &&
              !(ok = bar_wait(bar(L::kBarEmpty + slot), ((ring / L::kSlots) - 1) & 1, wc, 1)))
            break;
          int g;
          const int tile = tile_of_item(it, dual, i, g);
          const uint32_t dst = sbase + L::kOffKV + slot * L::kTile;
          const void* map = (i & 1) ? static_cast<const void*>(&p.tm_v)
                                    : static_cast<const void*>(&p.tm_k);
          if ((i & 1) && !dual) FA_TRACE_AT(i >> 1, 30);                // V_j issued
          if (!(i & 1) && !dual && i > 0) FA_TRACE_AT((i >> 1) - 1, 31);  // K_{j+1} issued
#ifdef FA_TRACE
          if (dual) FA_TRACE_AT((pc[g] + tile - (g ? it.jb[1] : it.jb[0])) & 63, (i & 1) ? 26 + g : 24 + g);
#endif
          ptx::mbar_arrive_expect_tx(bar(L::kBarFull + slot), L::kTile);
          const int row = it.ky + tile * kBlockN;
#pragma unroll
          for (int c = 0; c < L::kColBlocks; ++c) {
            if (p.ranges == 1)
              ptx::tma_load_3d(dst + c * L::kBlockBytes, map, bar(L::kBarFull + slot), c * 64,
                               it.kz, row, pol_kv);
            else
              ptx::tma_load_3d(dst + c * L::kBlockBytes, map, bar(L::kBarFull + slot), c * 64,
                               row, it.kz, pol_kv);
          }
        }
#ifdef FA_TRACE
        pc[0] += it.n_kv[0];
        pc[1] += it.n_kv[1];
#endif
      }
      // Drain: every copy this thread started must land before the CTA exits.
      for (int r = max(0, ring - L::kSlots); r < ring; ++r)
        bar_wait(bar(L::kBarFull + r % L::kSlots), (r / L::kSlots) & 1, wc, 2, false);
      for (int b = 0; b < 2; ++b)
        if (q_loads[b] > 0) bar_wait(bar(L::kBarQ + b), (q_loads[b] - 1) & 1, wc, 2, false);
    }
  } else if (warp == kWarpMma) {
    // ===================================================== MMA issuer
    // The whole warp runs this loop so that addresses and descriptors stay
    // warp-uniform; one elected lane issues each batch of tcgen05 ops.
    // This warp is on the critical path with few instructions to spare: one
    // tcgen05.mma holds the issuing thread ~50 cycles (measured on B200, for
    // N = 64 as for N = 128), and while the softmax warps of its
    // sub-partition run their exponential loops it gets few issue slots, so
    // every instruction costs several times its latency.  The loop therefore
    // keeps the waits' slow path out of line (bar_wait_lean), advances ring
    // slots and phases incrementally instead of dividing, and adds offsets to
    // the low word of the descriptors only.
    {
      constexpr uint32_t fmt = BF16 ? 1u : 0u;
      constexpr uint32_t idesc_qk = ptx::make_idesc_f16(kBlockM, kBlockN, fmt, 0, 0);
      constexpr uint32_t idesc_pv = ptx::make_idesc_f16(kBlockM, D, fmt, 0, 1);

      auto slot_of = [](int item) { return item % L::kSlots; };
      auto phase_of = [](int item) { return static_cast<uint32_t>((item / L::kSlots) & 1); };
      // Shared-memory descriptors of the slot-0 K tile (K-major), V tile
      // (MN-major) and the two Q tiles.  The start address sits in bits 0-13
      // of the low word and slot / K-step offsets never carry out of it
      // (shared memory < 256 KB), so offsets are added to the low word; the
      // high word (stride, version, swizzle) is the same for all four.
      const uint64_t k_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, 16, 1024);
      const uint64_t v_desc0 = ptx::smem_desc_sw128(sbase + L::kOffKV, L::kBlockBytes, 1024);
      const uint32_t d_hi = static_cast<uint32_t>(k_desc0 >> 32);
      const uint32_t k_lo0 = static_cast<uint32_t>(k_desc0);
      const uint32_t v_lo0 = static_cast<uint32_t>(v_desc0);
      const uint32_t q_lo0 = static_cast<uint32_t>(ptx::smem_desc_sw128(sbase + L::kOffQ, 16, 1024));
      const uint32_t q_lo1 =
          static_cast<uint32_t>(ptx::smem_desc_sw128(sbase + L::kOffQ + L::kTile, 16, 1024));
      constexpr uint32_t kSlotStep = L::kTile >> 4;
      // S_g = Q K^T with Q at descriptor low word q_lo and K in ring slot ks
      auto issue_s = [&](int g, int ks, uint32_t q_lo) {
        const uint32_t k_lo = k_lo0 + static_cast<uint32_t>(ks) * kSlotStep;
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = static_cast<uint32_t>(((kk / 4) * L::kBlockBytes + (kk % 4) * 32) >> 4);
            ptx::mma_ss(tmem + L::tS(g), ptx::make_desc(q_lo + off, d_hi),
                        ptx::make_desc(k_lo + off, d_hi), idesc_qk, kk > 0 ? 1u : 0u);
          }
          ptx::mma_commit(bar(L::kBarS + g));
        }
        __syncwarp();
      };
      auto commit = [&](uint32_t b) {
        if (ptx::elect_one()) ptx::mma_commit(b);
        __syncwarp();
      };
      auto wait = [&](uint32_t b, uint32_t ph, int site) {
        return __all_sync(0xffffffffu, bar_wait_lean(b, ph, wc, site));
      };
      // O_g (+)= P_g V with V in ring item `vi`; `first` starts the accumulator.
      // The PV steps on the announced early part of P (2 K-steps per quarter)
      // go out once the softmax has announced it (parity ph), the rest after
      // the whole P.
      auto issue_pv = [&](int g, int vs, bool first, uint32_t ph) -> bool {
        const uint32_t v_lo = v_lo0 + static_cast<uint32_t>(vs) * kSlotStep;
        if (!wait(bar(L::kBarPH + g), ph, 13 + 3 * g)) return false;
        ptx::tc_fence_after();
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 2 * kPEarlyQuarters; ++kk)
            ptx::mma_ts(tmem + L::tO(g), tmem + L::tP(g) + kk * 8,
                        ptx::make_desc(v_lo + kk * 128u, d_hi), idesc_pv,
                        (!first || kk > 0) ? 1u : 0u);
        }
        __syncwarp();
        if (!wait(bar(L::kBarP + g), ph, 13 + 3 * g)) return false;
        ptx::tc_fence_after();
        if (ptx::elect_one()) {
#pragma unroll
          for (int kk = 2 * kPEarlyQuarters; kk < kBlockN / 16; ++kk)
            ptx::mma_ts(tmem + L::tO(g), tmem + L::tP(g) + kk * 8,
                        ptx::make_desc(v_lo + kk * 128u, d_hi), idesc_pv, 1u);
          ptx::mma_commit(bar(L::kBarO + g));
        }
        __syncwarp();
        return true;
      };



      // Issue order per tile j (two groups g0, g1 ping-pong on the tensor pipe):
      //   PV0(j)  S0(j+1)  PV1(j)  S1(j+1)
      // so each group's softmax overlaps the other group's two MMAs.  S_g(j+1)
      // may overwrite P_g(j) (d=128): tcgen05.mma ops of one thread execute in
      // issue order, so PV_g(j) has read P_g(j) before S_g(j+1) writes it.
      // Work items: `ring` numbers K/V ring items across items, cnt[g] counts
      // the S/P/O completions of group g before the item (barrier parities).
      // A P arrival of group g for an item follows that group's reads of O
      // for the previous item, so the first PV of an item may overwrite O.
      bool ok = true;
      int ring = 0, k = 0;
      int cnt[2] = {0, 0};
      int qc[2] = {0, 0};  // shared mode: Q loads of group g before the item
      for (int w = w0; ok && w < n_work; w = consume_item(++k, ok, lane == 0)) {
        WorkItem it;
        decode_item(p, w, it);
        const int n_loop = it.n_loop;
        if (!dual) {
          // Q tiles in buffers 0 / 1; ring items numbered from `ring`, barrier
          // phases from cnt[g] and qc[g] (Q loads of group g so far), so a
          // persistent CTA walks several items.  A group without tiles in this
          // item issues nothing; with no tiles at all the producer loads no
          // K/V and this warp waits for nothing.  After an item's last S_g,
          // Q buffer g is released for the next item's Q tile.
          const bool g0 = it.n_kv[0] > 0;
          const bool g1 = it.n_kv[1] > 0;
          // ring position (slot, phase) of K_j, advanced item by item instead
          // of dividing the ring counter
          int ks = slot_of(ring);
          uint32_t kph = phase_of(ring);
          auto adv = [](int& sl, uint32_t& ph) {
            if (++sl == L::kSlots) {
              sl = 0;
              ph ^= 1u;
            }
          };
          if (n_loop > 0) {
            if (g0) ok = wait(bar(L::kBarQ), qc[0] & 1, 10);
            if (ok && g1) ok = wait(bar(L::kBarQ + 1), qc[1] & 1, 10);
            if (ok) ok = wait(bar(L::kBarFull + ks), kph, 11);
            if (ok) {
              if (g0) issue_s(0, ks, q_lo0);
              if (g1) issue_s(1, ks, q_lo1);  // K_0 is the item's first ring item
              commit(bar(L::kBarEmpty + ks));  // K0 read by both groups
              if (it.n_kv[0] == 1) commit(bar(L::kBarQFree));
              if (it.n_kv[1] == 1) commit(bar(L::kBarQFree + 1));
            }
          }
          for (int j = 0; ok && j < n_loop; ++j) {
            int vs = ks;  // V_j
            uint32_t vph = kph;
            adv(vs, vph);
            int ns = vs;  // K_{j+1}
            uint32_t nph = vph;
            adv(ns, nph);
            ks = ns;
            kph = nph;
            const bool next0 = j + 1 < it.n_kv[0];
            const bool next1 = j + 1 < it.n_kv[1];
            // V_j and K_{j+1} are waited for before the P waits, so that a
            // group's PV and next S go out back to back once its P is ready.
            // Every release the producer needs before loading them was
            // committed in an earlier iteration, so these waits cannot depend
            // on this one.
            if (lane == 0) FA_TRACE_AT(j, 6);
            if (!(ok = wait(bar(L::kBarFull + vs), vph, 12))) break;
            if ((next0 || next1) && !(ok = wait(bar(L::kBarFull + ns), nph, 14))) break;
            if (lane == 0) FA_TRACE_AT(j, 7);
            if (j < it.n_kv[0]) {
              if (lane == 0) FA_TRACE_AT(j, 0);
              if (!(ok = issue_pv(0, vs, j == 0, (cnt[0] + j) & 1))) break;
              if (lane == 0) FA_TRACE_AT(j, 4);
              if (next0) {
                if (lane == 0) FA_TRACE_AT(j, 1);
                issue_s(0, ns, q_lo0);
                if (lane == 0) FA_TRACE_AT(j, 5);
                if (j + 2 == it.n_kv[0]) commit(bar(L::kBarQFree));  // the item's last S0
                if (!next1) commit(bar(L::kBarEmpty + ns));
              }
            }
            if (j < it.n_kv[1]) {
              if (lane == 0) FA_TRACE_AT(j, 2);
              if (!(ok = issue_pv(1, vs, j == 0, (cnt[1] + j) & 1))) break;
            }
            commit(bar(L::kBarEmpty + vs));  // V_j read by both groups
            if (next1) {
              if (lane == 0) FA_TRACE_AT(j, 3);
              issue_s(1, ns, q_lo1);
              if (j + 2 == it.n_kv[1]) commit(bar(L::kBarQFree + 1));  // the item's last S1
              commit(bar(L::kBarEmpty + ns));
            }
          }
          if (g0) ++qc[0];
          if (g1) ++qc[1];
        } else {
          // Dual mode: each group streams its own K/V tiles (items from
          // k_item_of), so nothing waits for the other group's P; order per
          // iteration PV0(j) S0(j+1) PV1(j) S1(j+1), items released after use.
          // Both groups read Q buffer k & 1.
          const int qb = k & 1;
          const uint32_t q_lo = qb ? q_lo1 : q_lo0;
          if (n_loop > 0) {
            ok = wait(bar(L::kBarQ + qb), (k >> 1) & 1, 10);
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              if (!ok || it.n_kv[g] == 0) continue;
              const int ki = ring + k_item_of(it, true, g, 0);
              if (!(ok = wait(bar(L::kBarFull + slot_of(ki)), phase_of(ki), 11))) break;
              issue_s(g, slot_of(ki), q_lo);
              commit(bar(L::kBarEmpty + slot_of(ki)));
            }
          }
          for (int j = 0; ok && j < n_loop; ++j) {
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              if (j >= it.n_kv[g]) continue;
              const bool next = j + 1 < it.n_kv[g];
              const int vi = ring + k_item_of(it, true, g, j) + 1;
              const int ki = next ? ring + k_item_of(it, true, g, j + 1) : 0;
              if (!(ok = wait(bar(L::kBarFull + slot_of(vi)), phase_of(vi), 12))) break;
              if (next && !(ok = wait(bar(L::kBarFull + slot_of(ki)), phase_of(ki), 14))) break;
              if (lane == 0) FA_TRACE_AT((cnt[g] + j) & 63, 2 * g);  // V_j and K_{j+1} landed
              if (!(ok = issue_pv(g, slot_of(vi), j == 0, (cnt[g] + j) & 1))) break;
              if (lane == 0) FA_TRACE_AT((cnt[g] + j) & 63, 4 + g);  // P(j) seen, PV issued
              commit(bar(L::kBarEmpty + slot_of(vi)));
              if (next) {
                if (lane == 0) FA_TRACE_AT((cnt[g] + j) & 63, 1 + 2 * g);
                issue_s(g, slot_of(ki), q_lo);
                commit(bar(L::kBarEmpty + slot_of(ki)));
              }
            }
          }
          // Q buffer qb may be refilled once this item's MMAs have completed
          if (ok) commit(bar(L::kBarQFree + qb));
        }
        cnt[0] += it.n_kv[0];
        cnt[1] += it.n_kv[1];
        ring += it.n_items;
      }
      // Drain: all MMAs issued above complete before TMEM is released.
      commit(bar(L::kBarDrain));
      bar_wait(bar(L::kBarDrain), 0, wc, 19, false);
      __syncwarp();
    }
#ifdef FA_TRACE
   } else if (lane == 0 && !dual) {
    // trace observers: warp 10 (group 0) / 11 (group 1) timestamp the
    // completion of every S and PV MMA of their group
    // (polling without suspension, so the timestamps are not delayed by a
    // wake-up; each poll loop gives up after 2^26 polls or on abort)
    const int og = warp - kWarpMma - 1;
    auto poll = [&](uint32_t b, uint32_t ph) {
      for (uint32_t n = 0; n < (1u << 26); ++n) {
        if (ptx::mbar_test_wait(b, ph)) return true;
        if ((n & 1023u) == 1023u && *abort_flag) return false;
      }
      return false;
    };
    WorkItem it;  // shared mode: one work item per CTA
    decode_item(p, w0, it);
    for (int j = 0; j < it.n_kv[og]; ++j) {
      if (!poll(bar(L::kBarS + og), j & 1)) break;
      FA_TRACE_AT(j, 24 + 2 * og);
      if (!poll(bar(L::kBarO + og), j & 1)) break;
      FA_TRACE_AT(j, 25 + 2 * og);
    }
#endif
   }
  } else {
    // ===================================================== softmax groups
    ptx::setmaxnreg_inc<kRegsSoftmax>();
    const int sw = warp - kWarpSoftmax0;        // softmax warp 0..7
    const int g = sw >> 2;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;               // row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + L::tS(g);
    const uint32_t tP = tmem + lane_off + L::tP(g);
    const uint32_t tO = tmem + lane_off + L::tO(g);
    const float sl = p.scale_log2;
    bool ok = true;
    int cnt = 0;  // S / P / O completions of this group before the work item
    for (int round = 0, w = w0; ok && w < n_work; w = consume_item(++round, ok, true)) {
    WorkItem it;
    decode_item(p, w, it);
    const int n_tiles = g ? it.n_kv[1] : it.n_kv[0];
    const int jb = g ? it.jb[1] : it.jb[0];
    // global 128-row tile index
    const int tile = dual ? (p.dual == 2 ? it.qp : 2 * it.qp) : 2 * it.qp + g;
    const int q_row = tile * kBlockM + r;
    // key limit of this row: key k is visible iff k < row_end (causal:
    // pos + causal_off + 1; always at most nk)
    int row_end = it.nk;
    // smallest limit over the tile's rows: a K/V tile needs masking when any
    // of its keys lies at or beyond it
    int tile_end = it.nk;
    if (p.causal) {
      row_end = min(row_end, q_row % p.pos_mod + it.causal_off + 1);
      const int lo = tile * kBlockM;
      const int hi = min(lo + kBlockM - 1, it.nq - 1);
      const int min_pos = (p.pos_mod >= it.nq)                  ? lo
                          : (hi / p.pos_mod != lo / p.pos_mod) ? 0
                                                                : lo % p.pos_mod;
      tile_end = min(tile_end, min_pos + it.causal_off + 1);
    }

    float m = -INFINITY;  // running max of the scaled scores (log2 units)
    float l = 0.f;        // running sum of exp2(s - m)
    for (int j = 0; ok && j < n_tiles; ++j) {
      ok = __all_sync(0xffffffffu, bar_wait(bar(L::kBarS + g), (cnt + j) & 1, wc, 20 + g));
      if (!ok) break;
      if (lane == 0) FA_TRACE_AT(dual ? ((cnt + j) & 63) : j, 16 + sw);
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

      const int key0 = (jb + j) * kBlockN;
      const bool masked = key0 + kBlockN > tile_end;
      // Scaled tile maximum.  Unmasked tiles reduce the raw scores and scale
      // once (the exponent then folds scale and max into one packed FMA);
      // masked tiles are pre-scaled so that -inf marks excluded keys.
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

      if (r == 0) FA_TRACE_AT(dual ? ((cnt + j) & 63) : j, 28 + g);
      const float m_new = fmaxf(m, m_tile);
      const bool grow = m_new > m + kRescaleThreshold;
      if (j == 0) {
        m = m_new;
      } else {
        // O_g holds PV of tiles < j (their MMAs completed before S_g(j) was
        // signalled) and is not written again until this group arrives on P.
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? ptx::ex2_approx(m - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ptx::tmem_ld32(tO + c * 32, o);
            ptx::tmem_wait_ld();
            pin_after_wait<32>(o);
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              float a0 = __uint_as_float(o[i]), a1 = __uint_as_float(o[i + 1]);
              ptx::fmul2(a0, a1, a0, a1, alpha, alpha);
              o[i] = __float_as_uint(a0);
              o[i + 1] = __float_as_uint(a1);
            }
            ptx::tmem_st32(tO + c * 32, o);
          }
          ptx::tmem_wait_st();
          if (grow) l *= alpha;
        }
        if (grow) m = m_new;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;

      // P = exp2(x * sl_eff - m): packed FMA, then exp2 split between the MUFU
      // unit and a polynomial on the FMA pipe; written to TMEM in two halves.
      const uint32_t half_bar = bar(L::kBarPH + g);
      auto announce = [half_bar] { ptx::mbar_arrive(half_bar); };
      const float tile_sum = masked ? exp_tile<BF16, false>(x, sl_eff, neg_m, tP, announce)
                                    : exp_tile<BF16, true, kPairEmuPeriod<D>>(x, sl_eff, neg_m, tP, announce);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      if (lane == 0) FA_TRACE_AT(dual ? ((cnt + j) & 63) : j, 8 + sw);
      ptx::mbar_arrive(bar(L::kBarP + g));
      l += tile_sum;
    }

    // ---- epilogue: O / l -> global (or the split workspace), LSE
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    long long o_row0, lse_row0;
    int nq;
    item_out(p, w, o_row0, lse_row0, nq);
    const bool row_ok = q_row < nq;
    // split workspace row (the split modes have no row ranges: lse_row0 = bh*Nq)
    const size_t row_index = static_cast<size_t>(lse_row0) + q_row;
    T* const orow = reinterpret_cast<T*>(p.o) + o_row0 + static_cast<long long>(q_row) * p.o_rs;
    const long long lse_index = lse_row0 + q_row;
    if constexpr (D == 64) {
      if (p.dual == 2) {
        // Dual-tile item: the two groups hold O, m, l of the two halves of
        // the tile's keys on the same TMEM lanes.  Each thread publishes its
        // row's (m, l); after a named barrier over the eight softmax warps
        // (AND of their status, so a failed wait anywhere makes both groups
        // skip the output together) group g merges columns [32g, 32g + 32)
        //   O = (O0 2^(m0 - m) + O1 2^(m1 - m)) / (l0 2^(m0 - m) + l1 2^(m1 - m))
        // and group 0 writes the row's LSE.  A second barrier keeps either
        // group's next P (and so the next item's first PV, which overwrites
        // O) behind both groups' O reads.
        if (ok && n_tiles > 0)
          ok = __all_sync(0xffffffffu,
                          bar_wait(bar(L::kBarO + g), (cnt + n_tiles - 1) & 1, wc, 22 + g));
        float* xs = reinterpret_cast<float*>(smem + L::kOffXchg) + (round & 1) * (4 * kBlockM);
        xs[(g * kBlockM + r) * 2] = m;
        xs[(g * kBlockM + r) * 2 + 1] = l;
        const bool all_ok = ptx::bar_and(1, 256, ok);
        if (all_ok) {
          ptx::tc_fence_after();
          const int o_ = (g ^ 1) * kBlockM + r;
          const float m0 = g ? xs[2 * o_] : m, l0 = g ? xs[2 * o_ + 1] : l;
          const float m1 = g ? m : xs[2 * o_], l1 = g ? l : xs[2 * o_ + 1];
          const float mm = fmaxf(m0, m1);
          const float a0 = l0 > 0.f ? ptx::ex2_approx(m0 - mm) : 0.f;
          const float a1 = l1 > 0.f ? ptx::ex2_approx(m1 - mm) : 0.f;
          const float lsum = l0 * a0 + l1 * a1;
          const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
          // a group with key tiles has written all of its O rows (warp-uniform)
          const bool h0 = it.n_kv[0] > 0, h1 = it.n_kv[1] > 0;
          uint32_t u0[32] = {}, u1[32] = {};
          if (h0) ptx::tmem_ld32(tmem + lane_off + L::tO(0) + 32 * g, u0);
          if (h1) ptx::tmem_ld32(tmem + lane_off + L::tO(1) + 32 * g, u1);
          ptx::tmem_wait_ld();
          pin_after_wait<32>(u0);
          pin_after_wait<32>(u1);
          const float b0 = a0 * inv, b1 = a1 * inv;
          uint32_t hv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float v0 = 0.f, v1 = 0.f;
            if (h0) {
              v0 = __uint_as_float(u0[2 * i]) * b0;
              v1 = __uint_as_float(u0[2 * i + 1]) * b0;
            }
            if (h1) {
              v0 = fmaf(__uint_as_float(u1[2 * i]), b1, v0);
              v1 = fmaf(__uint_as_float(u1[2 * i + 1]), b1, v1);
            }
            hv[i] = pack2<BF16>(v0, v1);
          }
          if (row_ok) {
            uint4* dst = reinterpret_cast<uint4*>(orow + 32 * g);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(hv[4 * i], hv[4 * i + 1], hv[4 * i + 2], hv[4 * i + 3]);
            if (g == 0 && p.lse != nullptr)
              p.lse[lse_index] = lsum > 0.f ? (mm + __log2f(lsum)) * 0.69314718055994530942f
                                            : -INFINITY;
          }
        }
        ok = all_ok;
        ptx::tc_fence_before();
        ptx::bar_and(2, 256, true);
        cnt += n_tiles;
        continue;
      }
    }
    // partial-result slot of this group (split mode) in the workspace
    const int ws_slot = dual ? 2 * it.sp + g : it.sp;
    const bool partial = p.n_splits > 1 || dual;
    if (n_tiles == 0) {
      // No visible key for these rows (causal offset below zero): O = 0 and
      // LSE = -inf.  A split without tiles leaves the rows to other splits,
      // except the empty half of a dual split, whose slot the combine reads.
      if (dual && row_ok) p.ws_lse[static_cast<size_t>(ws_slot) * p.B * p.heads * p.Nq + row_index] = -INFINITY;
      if (!partial && row_ok) {
        uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
        if (p.lse != nullptr) p.lse[lse_index] = -INFINITY;
      }
    } else {
      if (ok)
        ok = __all_sync(0xffffffffu,
                        bar_wait(bar(L::kBarO + g), (cnt + n_tiles - 1) & 1, wc, 22 + g));
      if (ok) {
        ptx::tc_fence_after();
        const float inv_l = (l > 0.f) ? 1.0f / l : 0.f;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        const float lse_row = (l > 0.f) ? (m_use + __log2f(l)) * 0.69314718055994530942f : -INFINITY;
        if (!partial) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ptx::tmem_ld32(tO + c * 32, o);
            ptx::tmem_wait_ld();
            pin_after_wait<32>(o);
            uint32_t h[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              h[i] = pack2<BF16>(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
            if (row_ok) {
              uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                dst[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
            }
          }
          if (row_ok && p.lse != nullptr) p.lse[lse_index] = lse_row;
        } else {
          // partial result of this key split, normalised by its own row sum
          const size_t ws_row = static_cast<size_t>(ws_slot) * p.B * p.heads * p.Nq + row_index;
          float* wrow = p.ws_o + ws_row * D;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ptx::tmem_ld32(tO + c * 32, o);
            ptx::tmem_wait_ld();
            pin_after_wait<32>(o);
            if (row_ok) {
              float4* dst = reinterpret_cast<float4*>(wrow + c * 32);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l, __uint_as_float(o[4 * i + 1]) * inv_l,
                                     __uint_as_float(o[4 * i + 2]) * inv_l, __uint_as_float(o[4 * i + 3]) * inv_l);
            }
          }
          if (row_ok) p.ws_lse[ws_row] = lse_row;
        }
      }
    }
    cnt += n_tiles;
    }
  }

  // ---- teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) FA_TRACE_AT(kTraceTiles - 1, 31);  // CTA done
  if (warp == kWarpMma) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, L::kTmemCols);
  }
}

// Merge of key-split partial results: for each query row (one warp),
//   LSE = log sum_s exp(LSE_s),  O = sum_s exp(LSE_s - LSE) * O_s
// over the splits that hold data for the row's tile (the same count the
// attention kernel derives from kv_tiles_for_tile).  Rows without any
// visible key get O = 0 and LSE = -inf.
template <int D, bool BF16, int kBatch>
__global__ void __launch_bounds__(256) fa_combine_kernel(const __grid_constant__ FwdParams p) {
  constexpr int E = D / 32;  // elements per lane
  const long long n_rows = static_cast<long long>(p.B) * p.heads * p.Nq;
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const int lane = threadIdx.x & 31;
  // launched as a programmatic dependent of the attention kernel: the
  // partial results are complete and visible after this
  ptx::grid_dep_wait();
  const int q_row = static_cast<int>(row % p.Nq);
  const int total = kv_tiles_for_tile(p, q_row / kBlockM);
  // slots holding data: one per split with tiles (two in dual mode, where an
  // empty half stores LSE = -inf and no O)
  const int ns = min(p.n_splits, (total + p.tiles_per_split - 1) / p.tiles_per_split) *
                 (p.dual ? 2 : 1);
  // The slots' loads are independent: LSEs one per lane, then the O rows
  // kBatch at a time (16 for many splits, 8 for few, which keeps registers
  // and so occupancy up for many rows), so a row costs a few memory round
  // trips, not one per slot.
  float mx = -INFINITY;
  // first 32 slots' LSEs stay in registers for the weights
  const float ls0 = lane < ns ? p.ws_lse[static_cast<size_t>(lane) * n_rows + row] : -INFINITY;
  mx = ls0;
  for (int s = lane + 32; s < ns; s += 32) mx = fmaxf(mx, p.ws_lse[static_cast<size_t>(s) * n_rows + row]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  float wsum = 0.f;
  if (mx != -INFINITY) {
    for (int s0 = 0; s0 < ns; s0 += 32) {
      const int cnt = min(32, ns - s0);
      float w = 0.f;
      if (lane < cnt) {
        const float ls = s0 == 0 ? ls0 : p.ws_lse[static_cast<size_t>(s0 + lane) * n_rows + row];
        w = (ls == -INFINITY) ? 0.f : expf(ls - mx);
      }
      wsum += w;
      for (int i = 0; i < cnt; i += kBatch) {
        float ww[kBatch], v[kBatch][E];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          ww[u] = __shfl_sync(0xffffffffu, w, (i + u) & 31);
          if (i + u >= cnt) ww[u] = 0.f;
          const float* src =
              p.ws_o + (static_cast<size_t>(s0 + i + u) * n_rows + row) * D + lane * E;
          if (ww[u] != 0.f) {
            if constexpr (E == 4) {
              const float4 t = *reinterpret_cast<const float4*>(src);
              v[u][0] = t.x;
              v[u][1] = t.y;
              v[u][2] = t.z;
              v[u][3] = t.w;
            } else {
              const float2 t = *reinterpret_cast<const float2*>(src);
              v[u][0] = t.x;
              v[u][1] = t.y;
            }
          } else {
#pragma unroll
            for (int e = 0; e < E; ++e) v[u][e] = 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = fmaf(ww[u], v[u][e], acc[e]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
  }
  const float inv = wsum > 0.f ? 1.0f / wsum : 0.f;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  T* dst = reinterpret_cast<T*>(p.o) + row * D + lane * E;
  uint32_t h[E / 2];
#pragma unroll
  for (int e = 0; e < E / 2; ++e) h[e] = pack2<BF16>(acc[2 * e] * inv, acc[2 * e + 1] * inv);
  if constexpr (E == 4) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(h[0], h[1]);
  } else {
    *reinterpret_cast<uint32_t*>(dst) = h[0];
  }
  if (lane == 0 && p.lse != nullptr) p.lse[row] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
}

#include "fa_fwd_tile.cuh"
#include "fa_fwd_pair2.cuh"

}  // namespace

template <int D, bool BF16, int kSplit>
static cudaError_t launch_tile_impl(const FwdParams& p, int grid, cudaStream_t stream) {
  using C = tile::TCfg<kSplit>;
  auto kern = tile::fa_fwd_tile_kernel<D, BF16, kSplit>;
  constexpr int kSmem = tile::TLayout<D, kSplit>::kDynBytes;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    // a setmaxnreg split assumes exactly kLaunchRegs registers per thread
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    constexpr bool kSplitRegs = C::kRegsSoftmax != C::kLaunchRegs;
    if ((kSplitRegs && fa.numRegs != C::kLaunchRegs) || fa.numRegs > C::kLaunchRegs ||
        fa.maxThreadsPerBlock < C::kThreads)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  kern<<<grid, C::kThreads, kSmem, stream>>>(p);
  return cudaGetLastError();
}

template <int D, bool BF16>
static cudaError_t launch_tile(const FwdParams& p, int grid, cudaStream_t stream) {
  if (p.debug_flags & FA_DEBUG_TILE_SPLIT2) return launch_tile_impl<D, BF16, 2>(p, grid, stream);
  return launch_tile_impl<D, BF16, 4>(p, grid, stream);
}

template <bool BF16>
static cudaError_t launch_pair2_impl(const FwdParams& p, int n_clusters, cudaStream_t stream) {
  auto kern = pair2::fa_fwd_pair2_kernel<BF16>;
  constexpr int kSmem = pair2::PLayout::kDynBytes;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    // the setmaxnreg split assumes exactly kLaunchRegs registers per thread
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegs || fa.maxThreadsPerBlock < kThreads)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2u * static_cast<unsigned>(n_clusters));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int D, bool BF16>
static cudaError_t launch_impl(const FwdParams& p, int grid, cudaStream_t stream) {
  auto kern = fa_fwd_kernel<D, BF16>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    // The setmaxnreg split is only safe if the kernel is launched with exactly
    // kLaunchRegs registers per thread; anything else is refused.
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    if (fa.numRegs != kLaunchRegs || fa.maxThreadsPerBlock < kThreads)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Layout<D>::kDynBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_done[dev] = 1;
  }
  kern<<<grid, kThreads, Layout<D>::kDynBytes, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream) {
  const int n_all = p.n_qpairs * p.B * p.heads * p.n_splits;
  const int n_work = (p.item_end > 0 ? min(p.item_end, n_all) : n_all) - p.item0;
  if (n_work <= 0) return cudaSuccess;
  if (p.q_tile == 2) {  // CTA pairs, d = 128: one cluster per (batch*head, Q quad)
    if (head_dim != 128 || p.n_splits != 1 || p.dual || p.ranges) return cudaErrorInvalidValue;
    return bf16 ? launch_pair2_impl<true>(p, n_work, stream) : launch_pair2_impl<false>(p, n_work, stream);
  }
  if (p.q_tile) {
    if (head_dim == 64)
      return bf16 ? launch_tile<64, true>(p, n_work, stream) : launch_tile<64, false>(p, n_work, stream);
    return bf16 ? launch_tile<128, true>(p, n_work, stream) : launch_tile<128, false>(p, n_work, stream);
  }
  const int grid = (p.n_ctas > 0 && p.n_ctas < n_work) ? p.n_ctas : n_work;
  if (head_dim == 64) return bf16 ? launch_impl<64, true>(p, grid, stream) : launch_impl<64, false>(p, grid, stream);
  return bf16 ? launch_impl<128, true>(p, grid, stream) : launch_impl<128, false>(p, grid, stream);
}

// The combine is launched as a programmatic dependent of the attention
// kernel (which allows it early): its CTAs start while the attention kernel
// drains and wait in griddepcontrol.wait for its results.
#ifndef FA_COMBINE_PDL
#define FA_COMBINE_PDL 1
#endif
cudaError_t launch_combine(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream) {
  const long long n_rows = static_cast<long long>(p.B) * p.heads * p.Nq;
  const unsigned grid = static_cast<unsigned>((n_rows + 7) / 8);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = FA_COMBINE_PDL;
  const bool wide = p.n_splits * (p.dual ? 2 : 1) > 8;
  if (head_dim == 64) {
    if (wide)
      return bf16 ? cudaLaunchKernelEx(&cfg, fa_combine_kernel<64, true, 16>, p)
                  : cudaLaunchKernelEx(&cfg, fa_combine_kernel<64, false, 16>, p);
    return bf16 ? cudaLaunchKernelEx(&cfg, fa_combine_kernel<64, true, 8>, p)
                : cudaLaunchKernelEx(&cfg, fa_combine_kernel<64, false, 8>, p);
  }
  if (wide)
    return bf16 ? cudaLaunchKernelEx(&cfg, fa_combine_kernel<128, true, 16>, p)
                : cudaLaunchKernelEx(&cfg, fa_combine_kernel<128, false, 16>, p);
  return bf16 ? cudaLaunchKernelEx(&cfg, fa_combine_kernel<128, true, 8>, p)
              : cudaLaunchKernelEx(&cfg, fa_combine_kernel<128, false, 8>, p);
}

int smem_bytes_for(int head_dim) {
  return head_dim == 64 ? Layout<64>::kDynBytes : Layout<128>::kDynBytes;
}

cudaError_t read_status(unsigned long long* out, bool reset) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_fa_status, sizeof(*out));
  if (e != cudaSuccess) return e;
  if (reset) {
    const unsigned long long zero = 0ull;
    e = cudaMemcpyToSymbol(g_fa_status, &zero, sizeof(zero));
  }
  return e;
}

}  // namespace fa

// Decode and backward kernels (same translation unit: they share the device
// helpers above).
#include "fa_decode_sm100.cuh"
#include "fa_bwd_sm100.cuh"
