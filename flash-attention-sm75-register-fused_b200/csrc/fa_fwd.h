// Internal interface between the host C-ABI (fa_abi.cu) and the sm_100a
// kernel (fa_fwd_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "fa_b200.h"

namespace fa {

// Kernel parameters; passed by value as a __grid_constant__ so the TMA
// descriptors live in parameter space.
// Default size of the causal launch-order groups of heads (FwdParams::
// head_group).  Measured on B200: C4 causal +12 % against head-major order
// with groups of 8, +5 % with 4; fully pair-major order over C4's 64 heads
// loses the L2 sharing of K/V and was slower.
constexpr int kFwdHeadGroup = 8;

struct alignas(64) FwdParams {
  CUtensorMap tm_q;  // 3-D (d, Nq, B*heads), box (64, 128, 1), 128-byte swizzle
  CUtensorMap tm_k;  // 3-D (d, Nk, B*Hkv)
  CUtensorMap tm_v;  // 3-D (d, Nk, B*Hkv)
  void* o;           // [B*heads, Nq, d] f16/bf16 (packed varlen: [total_q, heads, d])
  int o_rs;          // elements between consecutive query rows of one head in O
  float* lse;        // [B*heads, Nq] fp32 or nullptr
  // Query rows are grouped as (batch*heads, Nq).  Unpacked: heads = Hq,
  // Nq = the query length.  GQA-packed (short queries): heads = Hkv and the
  // Nq = group*len rows of a KV head are the group's query heads one after
  // another (the same memory as [B, Hq, len, d]).
  int B, heads, Hkv, Nq, Nk;
  int group;         // query "heads" per KV head (1 when packed)
  int n_qpairs;      // Q units per (batch, head): ceil(Nq / 128) tiles (q_tile) or ceil(Nq / 256) pairs
  int q_tile;        // 1: the tile kernel (one 128-row Q tile per work item, S double-buffered);
                     // 0: the pair kernel (two Q tiles per item; dual mode);
                     // 2: the pair kernel on CTA pairs (d = 128; n_qpairs = 512-row quads)
  int n_kv_tiles;    // ceil(Nk / 128)
  int causal;        // key j visible to row r iff j <= pos(r) + causal_off
  int causal_off;
  int pos_mod;       // pos(r) = r % pos_mod (packed: the query length; else Nq)
  int n_splits;      // key-range splits per (batch*head, Q pair); 1 = no split
  int tiles_per_split;
  // dual = 1 (queries fit one 128-row tile): both softmax groups take the same
  // rows, group 0 the first half of the CTA's K/V tiles and group 1 the
  // second, each with its own K/V stream; every group writes a partial result
  // ("sub-split" 2*split + group) for the combine kernel.
  // dual = 2 (d = 64, no split): the same split of the keys for items of one
  // 128-row Q tile each (n_qpairs counts tiles); the groups merge their
  // halves inside the CTA and write O and LSE directly.
  int dual;
  int n_ctas;        // CTAs launched; 0 = one per work item, fewer = persistent CTAs
  // Causal item order: pair-major within groups of head_group (batch, head)
  // units, head-major across groups (>= 1; kFwdHeadGroup by default).
  int head_group;
  // Work items [item0, item_end) of the launch's item numbering (item_end 0:
  // all); a launch may cover a sub-range, e.g. the last items of a pair-kernel
  // launch handed to the tile kernel as twice as many one-tile items.
  int item0, item_end;
  // Persistent shared-mode launches (n_ctas > 0, dual = 0) with sched != 0:
  // rounds >= sched_round take their items from a device-wide counter (slot
  // sched % kSchedSlots, tagged with sched) instead of the boustrophedon
  // deal, so the CTAs that drew lighter items take more of the last ones.
  unsigned sched;
  int sched_round;
  float* ws_o;       // partial O [n_splits * (1 + dual)][B*heads][Nq][d] fp32 (normalised)
  float* ws_lse;     // partial LSE [n_splits * (1 + dual)][B*heads][Nq] (natural log)
  float scale_log2;  // scale * log2(e)
  // Per-batch row ranges (ranges != 0; no packing, split or dual mode then).
  // Sequence b's queries are rows [q_lo[b], q_hi[b]) and its keys rows
  // [k_lo[b], k_hi[b]); Nq / Nk are the largest lengths (they size the grid).
  //   ranges = 1, packed varlen: Q/O [total_q, heads, d], K/V [total_k, Hkv, d]
  //     (maps (d, H, T), box (64, 1, 128)); q_lo = cu_seqlens_q, q_hi =
  //     cu_seqlens_q + 1; LSE [heads, q_lim]; causal_off is added to the
  //     per-sequence offset nk - nq (bottom-right) or 0 (top-left), chosen by
  //     causal_br.
  //   ranges = 2, padded batch: the fixed [B, heads, N, d] layout with valid
  //     rows [lo, hi) per batch entry; the causal rule stays that of the full
  //     padded rows (key j visible to row i iff j <= i + causal_off).
  // Rows outside a sequence's range are not written.
  // Rows are clamped to [0, q_lim) / [0, k_lim) (packed: total_q / total_k,
  // padded: Nq / Nk), so no range reaches outside the tensors.  Query rows of
  // a sequence past the grid's 256*n_qpairs rows are not computed.
  int ranges;
  int causal_br;
  int q_lim, k_lim;
  const int* q_lo;
  const int* q_hi;
  const int* k_lo;
  const int* k_hi;
  int debug_flags;
  long long* trace;  // timeline samples, used only in FA_TRACE builds
  unsigned epoch;    // launch counter, tags device status words
  unsigned long long timeout_ns;
};

// Number of K/V tiles a 128-row query tile t needs (all tiles when not causal).
// Shared by the attention kernel and the split combine so that both agree on
// which splits hold data for a row.
// nq query rows, n_kv K/V tiles, key j visible to row r iff
// j <= r % pos_mod + causal_off (causal).  Tiles past the last row need none.
__host__ __device__ inline int kv_tiles_core(int causal, int nq, int n_kv, int causal_off,
                                             int pos_mod, int t) {
  const int lo = t * 128;
  if (lo >= nq) return 0;
  if (!causal) return n_kv;
  const int hi = (lo + 127 < nq - 1) ? lo + 127 : nq - 1;
  int max_pos;
  if (pos_mod >= nq) {
    max_pos = hi;
  } else {
    max_pos = (hi / pos_mod != lo / pos_mod) ? pos_mod - 1 : hi % pos_mod;
  }
  const long long kmax = static_cast<long long>(max_pos) + causal_off;  // last visible key
  if (kmax < 0) return 0;
  const long long n = kmax / 128 + 1;
  return n < n_kv ? static_cast<int>(n) : n_kv;
}

__host__ __device__ inline int kv_tiles_for_tile(const FwdParams& p, int t) {
  return kv_tiles_core(p.causal, p.Nq, p.n_kv_tiles, p.causal_off, p.pos_mod, t);
}

// Backward parameters (dK/dV and dQ kernels).  Q, K, V, dO as 3-D TMA maps
// like the forward; l2 / dd hold per query row -LSE*log2(e) (-inf past N) and
// -rowsum(dO * O) (0 past N), each [B*Hq][n_pad] with n_pad = 128 * n_tiles.
struct alignas(64) BwdParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_do;
  void* dq;          // [B, Hq, N, d]
  void* dk;          // [B, Hkv, N, d]
  void* dv;          // [B, Hkv, N, d]
  const float* l2;
  const float* dd;
  // Per (batch*Hq, query tile): two 4 KB K-major operand tiles (128 query rows
  // x 16 f16/bf16, no swizzle, 8x16-byte core matrices 128 B apart along K and
  // 256 B apart along rows): row n holds -LSE/scale, then -D, each as three
  // 16-bit terms (k = 0..2) summing to the fp32 value.  Multiplied by a tile
  // of ones, they pre-load the S^T and dP^T accumulators of the dK/dV kernel.
  const uint8_t* vt;
  // Padded batch (all non-null) or nullptr: batch entry b's valid query rows
  // are [q_lo[b], q_hi[b]) and valid keys [k_lo[b], k_hi[b]) (int32 device
  // arrays, clamped to [0, N]); outside them P = 0, so invalid keys get
  // dK = dV = 0 and invalid query rows dQ = 0.
  const int* q_lo;
  const int* q_hi;
  const int* k_lo;
  const int* k_hi;
  // Packed variable-length batch (self-attention): cu_seqlens [B + 1] or
  // nullptr.  Sequence b owns rows [cu[b], cu[b+1]) of Q, K, V, O, dO, dQ, dK,
  // dV ([total, H, d]; maps (d, H, T)) and LSE [Hq, total]; N is the longest
  // sequence (it sizes the grid and the per-tile workspace).
  const int* cu;
  int total;
  int B, Hq, Hkv, N, n_pad, group, n_tiles, causal;
  float scale, scale_log2;
  long long* trace;  // timeline samples, used only in FA_TRACE builds
  unsigned epoch;
  unsigned long long timeout_ns;
};

cudaError_t launch_fwd(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream);
// Decode kernel (at most 16 query rows per batch*head, dual = 0): one pass
// over the (batch*head, key split) items; partial results for the combine
// when n_splits > 1.
cudaError_t launch_decode(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream);
// dD / L2 preprocessing (reads O, dO, LSE) and the two backward kernels.
cudaError_t launch_bwd(const BwdParams& p, const void* o, const void* dout, const float* lse,
                       int head_dim, bool bf16, cudaStream_t stream);
int bwd_smem_bytes_for(int head_dim);
// Merges the n_splits partial results of p.ws_o / p.ws_lse into p.o / p.lse.
cudaError_t launch_combine(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream);
int smem_bytes_for(int head_dim);
cudaError_t read_status(unsigned long long* out, bool reset);

}  // namespace fa
