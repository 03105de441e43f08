// Host side of the C ABI declared in include/fa_b200.h: argument checks,
// TMA descriptor construction, launch of the sm_100a kernel, the
// reference-compatible blocking launchers, and the materialised ("naive")
// attention that the reference exports for API completeness.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "fa_b200.h"
#include "fa_fwd.h"

namespace {

std::atomic<unsigned> g_epoch{1};
// Numbers of persistent launches with dynamically dealt last rounds (never 0:
// a counter slot tagged 0 is unused).
std::atomic<unsigned> g_sched{1};
unsigned next_sched() {
  const unsigned v = g_sched.fetch_add(1, std::memory_order_relaxed);
  return v != 0u ? v : g_sched.fetch_add(1, std::memory_order_relaxed);
}
std::atomic<unsigned long long> g_timeout_ns{1000000000ull};
std::atomic<int> g_debug_flags{0};
std::atomic<long long*> g_trace{nullptr};

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Encoded tensor maps of recent calls: a map is a pure function of its
// arguments, so a call that repeats (pointer, shape, dtype, box) -- every
// layer of a model, every benchmark step -- reuses the encoding instead of
// paying the driver's encoder again.  Direct-mapped, guarded by a mutex.
struct MapKey {
  const void* base;
  long long n, bh;
  int d, box_rows, bf16, kind;
  bool operator==(const MapKey& o) const {
    return base == o.base && n == o.n && bh == o.bh && d == o.d && box_rows == o.box_rows &&
           bf16 == o.bf16 && kind == o.kind;
  }
};
constexpr int kMapCacheSize = 64;
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool valid;
};
std::mutex g_map_mu;
MapEntry g_map_cache[kMapCacheSize];

int map_slot(const MapKey& k) {
  uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
  h ^= static_cast<uint64_t>(k.n) * 0xC2B2AE3D27D4EB4Full + static_cast<uint64_t>(k.bh) * 31 +
       static_cast<uint64_t>(k.d * 7 + k.box_rows * 13 + k.bf16 * 3 + k.kind);
  return static_cast<int>((h >> 32) % kMapCacheSize);
}

bool cached_map(CUtensorMap* map, const MapKey& k) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  const MapEntry& e = g_map_cache[map_slot(k)];
  if (!e.valid || !(e.key == k)) return false;
  *map = e.map;
  return true;
}

void remember_map(const CUtensorMap& map, const MapKey& k) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  MapEntry& e = g_map_cache[map_slot(k)];
  e.key = k;
  e.map = map;
  e.valid = true;
}

// [rows = B*H*N, d] tensor viewed as 3-D (d, N, B*H) so that a box of
// `box_rows` rows never crosses into the next head: rows >= N read as zeros.
bool make_map(CUtensorMap* map, const void* base, int d, int n, long long bh, bool bf16,
              unsigned box_rows = 128) {
  const MapKey key{base, n, bh, d, static_cast<int>(box_rows), bf16 ? 1 : 0, 0};
  if (cached_map(map, key)) return true;
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(n),
                              static_cast<cuuint64_t>(bh)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2,
                                 static_cast<cuuint64_t>(n) * static_cast<cuuint64_t>(d) * 2};
  const cuuint32_t box[3] = {64, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r =
      fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  remember_map(*map, key);
  return true;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuCtxGetCurrent_v4000 ctx_get_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(ptr);
  });
  return fn;
}

// Checks that the current device is an sm_100 part and that its primary
// context is current on the calling thread.  The tensor-map encoder is a
// driver call that needs a current context, and a thread that has only
// touched cached allocations (PyTorch's autograd worker, a fresh host
// thread) may not have one yet; cudaSetDevice binds the primary context.
int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_CUDA;
  CUcontext ctx = nullptr;
  const auto get_ctx = ctx_get_fn();
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
    if (cudaSetDevice(dev) != cudaSuccess) return FA_ERR_CUDA;
  }
  static int major_cache[64] = {0};
  int major = (dev >= 0 && dev < 64) ? major_cache[dev] : 0;
  if (major == 0) {
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return FA_ERR_CUDA;
    if (dev >= 0 && dev < 64) major_cache[dev] = major;
  }
  return major == 10 ? FA_OK : FA_ERR_DEVICE;
}

// ------------------------------------------------------------------ naive
// S = Q K^T * scale (masked entries = -1e9, as reference naive_attention.cu:31-34),
// row softmax in place, O = P V.  One thread per output element; fp32 math.
__global__ void naive_qk_kernel(const __half* __restrict__ Q, const __half* __restrict__ K,
                                float* __restrict__ S, int n, int d, float scale, int causal) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;  // key
  const int i = blockIdx.y * blockDim.y + threadIdx.y;  // query
  const long long bh = blockIdx.z;
  if (i >= n || j >= n) return;
  float* out = S + (bh * n + i) * static_cast<long long>(n) + j;
  if (causal && j > i) {
    *out = -1e9f;
    return;
  }
  const __half* q = Q + (bh * n + i) * d;
  const __half* k = K + (bh * n + j) * d;
  float acc = 0.f;
  for (int c = 0; c < d; ++c) acc = fmaf(__half2float(q[c]), __half2float(k[c]), acc);
  *out = acc * scale;
}

__global__ void naive_softmax_kernel(float* __restrict__ S, int n) {
  // one warp per row
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const long long bh = blockIdx.y;
  if (row >= n) return;
  float* s = S + (bh * n + row) * static_cast<long long>(n);
  float mx = -INFINITY;
  for (int c = lane; c < n; c += 32) mx = fmaxf(mx, s[c]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int c = lane; c < n; c += 32) {
    const float e = expf(s[c] - mx);
    s[c] = e;
    sum += e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.0f / sum;
  for (int c = lane; c < n; c += 32) s[c] *= inv;
}

__global__ void naive_pv_kernel(const float* __restrict__ P, const __half* __restrict__ V,
                                __half* __restrict__ O, int n, int d) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;  // head-dim column
  const int i = blockIdx.y * blockDim.y + threadIdx.y;  // query
  const long long bh = blockIdx.z;
  if (i >= n || c >= d) return;
  const float* p = P + (bh * n + i) * static_cast<long long>(n);
  const __half* v = V + bh * n * static_cast<long long>(d) + c;
  float acc = 0.f;
  for (int j = 0; j < n; ++j) acc = fmaf(p[j], __half2float(v[static_cast<long long>(j) * d]), acc);
  O[(bh * n + i) * d + c] = __float2half_rn(acc);
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  static std::atomic<int> cache[64];
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// How one call is laid out on the GPU.  Short GQA queries (Nq <= 128) are
// "packed": the group's query heads are consecutive in [B, Hq, Nq, d], so the
// G*Nq rows of one KV head form one row sequence (pos = row % Nq) and share
// every K/V tile.  When (batch*head, Q pair) units alone fill less than one
// wave and a workspace is available, the key range is split so that about two
// CTAs per SM run; a combine kernel merges the splits.
struct Plan {
  bool pack = false;
  bool decode = false;  // at most 16 query rows: the decode kernel
  bool dual = false;  // one Q tile: the two softmax groups split the key tiles
  int n_ctas = 0;     // persistent CTAs (dual mode), 0 = one per work item
  bool q_tile = true;  // the tile kernel (else the pair kernel)
  bool pair2 = false;  // the pair kernel on CTA pairs (n_qpairs counts 512-row quads)
  int heads = 0, rows = 0, group = 1, pos_mod = 1, n_qpairs = 0, n_kv_tiles = 0;
  int n_splits = 1, tiles_per_split = 0;
  size_t ws_o_bytes = 0, ws_bytes = 0;
};

constexpr int kDecodeRows = 16;  // query rows of the decode kernel's blocks

// Kernel choice for a launch whose pair kernel would have `pair_units` work
// items (measured on B200: the tile kernel is faster only while the pair
// kernel leaves SMs idle in its single wave, e.g. 10.6 vs 17.1 us at
// B=1 H=1 N=512; from C2 to C5 the pair kernel is 3-30 % faster).
// FA_DEBUG_PAIR_KERNEL / FA_DEBUG_TILE_KERNEL force one of them.
bool use_tile_kernel(long long pair_units) {
  const int flags = g_debug_flags.load(std::memory_order_relaxed);
  if (flags & (FA_DEBUG_PAIR_KERNEL | FA_DEBUG_PAIR2_KERNEL)) return false;
  if (flags & FA_DEBUG_TILE_KERNEL) return true;
  return pair_units < sm_count();
}

// The pair kernel on CTA pairs (fa_fwd_pair2: each product issued once for
// two SMs, each SM streaming half of every K/V tile) applies to d = 128 over
// plain rows (no GQA packing, more than one tile of queries).  It is opt-in
// (FA_DEBUG_PAIR2_KERNEL): measured on B200 against the one-SM pair kernel
// on one box, C5 1110-1129 vs 1129-1136 TFLOPS and C4 GQA causal 923 vs
// 1034 (a causal group computes its extra diagonal tile for both CTAs).
bool use_pair2_kernel(bool /*tile*/, int d, bool packed, int rows) {
  const int flags = g_debug_flags.load(std::memory_order_relaxed);
  if (d != 128 || packed || rows <= 128) return false;
  return (flags & FA_DEBUG_PAIR2_KERNEL) != 0;
}

Plan make_plan(int B, int Hq, int Hkv, int Nq, int Nk, int d, bool allow_split) {
  Plan k;
  const int G = Hq / Hkv;
  k.pack = G > 1 && Nq <= 128;
  k.heads = k.pack ? Hkv : Hq;
  k.rows = k.pack ? G * Nq : Nq;
  k.group = k.pack ? 1 : G;
  k.pos_mod = k.pack ? Nq : k.rows;
  // Square and chunked prefill run the pair kernel (two 128-row Q tiles per
  // work item) unless its work items would not fill one wave of SMs; then
  // the tile kernel (one tile per item) doubles the CTAs.  Dual and decode
  // launches have one unit per row block either way.
  // (with a workspace, an under-filled launch is split along the keys
  // instead, which measured faster on the pair kernel: a 512-query causal
  // chunk of an 8192-key cache 86-101 us against 151 us on the tile kernel)
  k.q_tile = !allow_split &&
             use_tile_kernel(static_cast<long long>((k.rows + 255) / 256) * B * k.heads);
  k.pair2 = use_pair2_kernel(k.q_tile, d, k.pack, k.rows);
  k.n_qpairs = k.q_tile  ? (k.rows + 127) / 128
               : k.pair2 ? (k.rows + 511) / 512
                         : (k.rows + 255) / 256;
  k.n_kv_tiles = (Nk + 127) / 128;
  k.tiles_per_split = k.n_kv_tiles;
  const long long units = static_cast<long long>(k.n_qpairs) * B * k.heads;
  const int sms = sm_count();
  // (CTA pairs are only chosen when the pair kernel's units fill a wave, so
  // they never split)
  if (allow_split && !k.pair2 && units < sms && k.n_kv_tiles > 1) {
    // One CTA per (unit, split): pick the balanced split with the fewest
    // waves x (tiles per split + start-up), a CTA's start-up (first loads,
    // epilogue, its share of the combine) counted as 4 tiles, at least two
    // splits.  Measured on 512- and 256-query chunks: 1.4x and 1.1x faster
    // than about two CTAs per SM, whose 2.2 waves left most SMs idle in the
    // last; a start-up of 1-2 tiles chose many short splits for a
    // 1024-query chunk (15 % slower), 4 matches the old plan there.
    constexpr long long kStartTiles = 4;
    const long long n = k.n_kv_tiles;
    long long best_tps = (n + 1) / 2, best_cost = -1;
    for (long long tps = 1; tps < n; ++tps) {
      const long long ns = (n + tps - 1) / tps;
      if (ns > 64 || (n + ns - 1) / ns != tps) continue;
      const long long waves = (units * ns + sms - 1) / sms;
      const long long cost = waves * (tps + kStartTiles);
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best_tps = tps;
      }
    }
    k.tiles_per_split = static_cast<int>(best_tps);
    k.n_splits = static_cast<int>((n + best_tps - 1) / best_tps);
  }
  // Queries that fit one 128-row tile leave the CTA's second softmax group
  // idle; in dual mode the two groups take halves of the CTA's key tiles.
  // Dual launches are persistent: one CTA per SM walks work items of an even
  // number of key tiles, so no wave tail remains and the ring prefetches the
  // next item's tiles during the current one.
  k.dual = allow_split && k.rows <= 128 && k.n_kv_tiles >= 2;
  if (k.dual) {
    // about six work items per persistent CTA (measured: 3 was slower on the
    // decode workloads of bench.py, 1-2 leave a wave tail or unbalanced items)
    constexpr long long kItemsPerCta = 6;
    const long long tiles = units * k.n_kv_tiles;
    const long long per = kItemsPerCta * sms;
    long long tps = (tiles + per - 1) / per;
    if (tps < 2) tps = 2;
    // at most 32 splits per row keep the combine short
    if (tps * 32 < k.n_kv_tiles) tps = (k.n_kv_tiles + 31) / 32;
    if (tps > k.n_kv_tiles) tps = k.n_kv_tiles;
    // balance: the same number of tiles (+-2) in every split of a row
    const long long ns = (k.n_kv_tiles + tps - 1) / tps;
    tps = (k.n_kv_tiles + ns - 1) / ns;
    tps += tps & 1;
    if (tps > k.n_kv_tiles) tps = k.n_kv_tiles;
    k.tiles_per_split = static_cast<int>(tps);
    k.n_splits = (k.n_kv_tiles + k.tiles_per_split - 1) / k.tiles_per_split;
    const long long n_work = units * k.n_splits;
    k.n_ctas = static_cast<int>(n_work < sms ? n_work : sms);
  }
  // At most 16 query rows per (batch, head) -- decode -- run the decode
  // kernel (keys on the MMA's M dimension, persistent CTAs walking (head, key
  // split) items).  The split is chosen for balance: fewest waves of items
  // over the SMs, each item costing its tiles plus about half a tile of
  // hand-off; at most 64 splits per row keep the combine short.  Splits count
  // 128-key tiles also at d = 64, where the kernel's tiles are 256 keys.
  k.decode = k.rows <= kDecodeRows;
  if (k.decode) {
    k.dual = false;
    const long long n = k.n_kv_tiles;
    long long best_tps = n, best_cost = -1;
    if (allow_split) {
      for (long long tps = 1; tps <= n; ++tps) {
        const long long ns = (n + tps - 1) / tps;
        if (ns > 64 || (n + ns - 1) / ns != tps) continue;  // balanced splits only
        // d = 64 tiles are 256 keys: splits start on a 256-key boundary
        if (d == 64 && (tps & 1) && tps != n) continue;
        const long long waves = (units * ns + sms - 1) / sms;
        const long long cost = waves * (2 * tps + 1);
        if (best_cost < 0 || cost < best_cost) {
          best_cost = cost;
          best_tps = tps;
        }
      }
    }
    k.tiles_per_split = static_cast<int>(best_tps);
    k.n_splits = static_cast<int>((n + best_tps - 1) / best_tps);
    const long long n_work = units * k.n_splits;
    k.n_ctas = static_cast<int>(n_work < sms ? n_work : sms);
  }
  // Pair-kernel launches of many waves run persistent CTAs, one per SM: a
  // CTA's next item starts its loads and first products while the current
  // item's last tiles and epilogue finish.  Items are dealt out statically,
  // so with few rounds uneven (causal) items leave some CTAs idle at the end
  // that hardware scheduling of one CTA per item would have kept busy:
  // measured on B200, C5 +2-4 % and C5 causal +3-7 % (27.7 rounds), C4 GQA
  // causal -4 % (6.9 rounds), a causal 16-head N=8192 launch -25 % (3.5
  // rounds); hence at least 16 rounds.
  if (!k.dual && !k.decode && !k.q_tile && !k.pair2 && k.n_splits == 1 &&
      (g_debug_flags.load(std::memory_order_relaxed) & FA_DEBUG_NO_PERSIST) == 0) {
    constexpr long long kMinRounds = 16;
    const long long n_work = static_cast<long long>(k.n_qpairs) * B * k.heads;
    if (n_work >= kMinRounds * sms) k.n_ctas = sms;
  }
  if (k.n_splits > 1 || k.dual) {
    const size_t slots = static_cast<size_t>(k.n_splits) * (k.dual ? 2 : 1);
    const size_t rows_total = static_cast<size_t>(B) * k.heads * k.rows;
    k.ws_o_bytes = slots * rows_total * d * sizeof(float);
    k.ws_bytes = k.ws_o_bytes + slots * rows_total * sizeof(float);
  }
  return k;
}

// Shared argument checks of fa_fwd / fa_fwd_kvcache; FA_OK means "launch".
// *empty is set when there is nothing to compute.
int check_args(const void* Q, const void* K, const void* V, const void* O, const float* lse,
               int B, int Hq, int Hkv, int Nq, int Nk, int head_dim, float scale, int causal,
               int dtype, bool* empty) {
  *empty = false;
  if (B < 0 || Hq < 0 || Hkv < 0 || Nq < 0 || Nk < 0) return FA_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_DTYPE;
  if (causal < FA_CAUSAL_NONE || causal > FA_CAUSAL_TOP_LEFT) return FA_ERR_INVALID_ARG;
  if (B == 0 || Hq == 0 || Nq == 0) {
    *empty = true;
    return FA_OK;
  }
  if (Hkv == 0 || Nk == 0) return FA_ERR_INVALID_ARG;
  if (Hq % Hkv != 0) return FA_ERR_GQA_DIVISIBILITY;
  if (!Q || !K || !V || !O) return FA_ERR_INVALID_ARG;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) ||
      (reinterpret_cast<uintptr_t>(lse) & 3u))
    return FA_ERR_ALIGNMENT;
  if (!std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  const long long rows = static_cast<long long>(B) * Hq * Nq;
  if (Nq > (1 << 30) || Nk > (1 << 30) || rows > (1LL << 40) ||
      static_cast<long long>(B) * Hq * ((static_cast<long long>(Nq) + 127) / 128) > 0x7fffffffLL)
    return FA_ERR_TOO_LARGE;
  return check_device();
}

int launch_attention(const void* Q, const void* K, const void* V, void* O, float* lse, int B,
                     int Hq, int Hkv, int Nq, int Nk, int head_dim, float scale, int causal,
                     int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  const bool bf16 = dtype == FA_DTYPE_BF16;
  Plan k = make_plan(B, Hq, Hkv, Nq, Nk, head_dim, workspace != nullptr);
  const bool partial = k.n_splits > 1 || k.dual;
  if (partial && (workspace_bytes < k.ws_bytes || !aligned16(workspace)))
    k = make_plan(B, Hq, Hkv, Nq, Nk, head_dim, false);  // too small: no split
  if (static_cast<long long>(k.n_qpairs) * B * k.heads * k.n_splits > 0x7fffffffLL)
    return FA_ERR_TOO_LARGE;

  fa::FwdParams p;
  const long long bh = static_cast<long long>(B) * k.heads;
  // the decode kernel's K/V tiles are 256 keys at d = 64 (32 KB, like d = 128)
  const unsigned kv_box = (k.decode && head_dim == 64) ? 256 : 128;
  // CTA pairs load half of a K tile (64 keys) per CTA
  const unsigned k_box = k.pair2 ? 64 : kv_box;
  if (!make_map(&p.tm_q, Q, head_dim, k.rows, bh, bf16, k.decode ? kDecodeRows : 128) ||
      !make_map(&p.tm_k, K, head_dim, Nk, static_cast<long long>(B) * Hkv, bf16, k_box) ||
      !make_map(&p.tm_v, V, head_dim, Nk, static_cast<long long>(B) * Hkv, bf16, kv_box))
    return FA_ERR_TENSOR_MAP;
  p.o = O;
  p.o_rs = head_dim;
  p.lse = lse;
  p.ranges = 0;
  p.causal_br = 0;
  p.q_lim = p.k_lim = 0;
  p.q_lo = p.q_hi = p.k_lo = p.k_hi = nullptr;
  p.B = B;
  p.heads = k.heads;
  p.Hkv = Hkv;
  p.Nq = k.rows;
  p.Nk = Nk;
  p.group = k.group;
  p.n_qpairs = k.n_qpairs;
  p.q_tile = (k.q_tile && !k.dual && !k.decode) ? 1 : (k.pair2 && !k.dual && !k.decode) ? 2 : 0;
  p.n_kv_tiles = k.n_kv_tiles;
  p.causal = causal != FA_CAUSAL_NONE ? 1 : 0;
  p.causal_off = causal == FA_CAUSAL_BOTTOM_RIGHT ? Nk - Nq : 0;
  p.pos_mod = k.pos_mod;
  p.n_splits = k.n_splits;
  p.tiles_per_split = k.tiles_per_split;
  p.dual = k.dual ? 1 : 0;
  p.n_ctas = k.n_ctas;
  // A d = 64 launch of more than one and at most two waves of pair items
  // also runs persistent CTAs: the second item of a CTA loads while its
  // first finishes, instead of a fresh CTA starting up in the second wave;
  // causal items (heaviest first) are dealt boustrophedon-wise, so a CTA's
  // second item is one of the lightest (measured on B200: C2, 192 items,
  // 342-345 -> 349-357 TFLOPS; C3 causal, 256 items, 417 -> 433;
  // non-causal launches of 3.5 and 6.9 rounds measured no gain or a loss).
  if (head_dim == 64 && p.n_ctas == 0 && !k.dual && !k.decode && !k.q_tile &&
      !k.pair2 && k.n_splits == 1 &&
      (g_debug_flags.load(std::memory_order_relaxed) & FA_DEBUG_NO_PERSIST) == 0) {
    const long long n_items = static_cast<long long>(k.n_qpairs) * B * k.heads;
    const int sms = sm_count();
    if (n_items > sms && n_items <= 2LL * sms) p.n_ctas = sms;
  }
  // Dual-tile items (d = 64, square launches): one 128-row Q tile per item,
  // its key tiles split between the two softmax groups and merged inside the
  // CTA, on persistent CTAs.  Finer items than Q pairs, shorter ones than the
  // tile kernel's: C2's 192 pair items (1.3 waves, two items on 44 CTAs)
  // become 384 half-length items (2.6 waves).  By default for non-causal
  // launches of at most two waves of Q pairs (measured on B200: C2 348 ->
  // 371 TFLOPS against persistent Q pairs; against the tile kernel below one
  // wave, C1 5.9 -> 6.5, B=1 H=4 N=4096 382 -> 495, B=1 H=8 N=512 44 -> 50,
  // B=2 H=8 N=1024 262 -> 267); causal items stay on Q pairs (C3 430 -> 348
  // with dual tiles).  FA_DEBUG_DUAL_TILES forces them wherever they apply,
  // FA_DEBUG_PAIR_KERNEL / FA_DEBUG_TILE_KERNEL keep their kernels.
  const unsigned dbg = static_cast<unsigned>(g_debug_flags.load(std::memory_order_relaxed));
  const long long pair_items = static_cast<long long>((k.rows + 255) / 256) * B * k.heads;
  const bool dual_tiles_default =
      p.causal == 0 && pair_items <= 2LL * sm_count() &&
      (dbg & (FA_DEBUG_PAIR_KERNEL | FA_DEBUG_TILE_KERNEL | FA_DEBUG_PAIR2_KERNEL)) == 0;
  if (((dbg & FA_DEBUG_DUAL_TILES) != 0 || dual_tiles_default) && head_dim == 64 && !k.dual &&
      !k.decode && !k.pair2 && k.n_splits == 1 && k.heads == Hq && Nq == Nk &&
      k.n_kv_tiles >= 2) {
    p.q_tile = 0;
    p.dual = 2;
    p.n_qpairs = (k.rows + 127) / 128;
    const long long items = static_cast<long long>(p.n_qpairs) * B * k.heads;
    const int sms = sm_count();
    p.n_ctas = items < sms ? static_cast<int>(items) : sms;
  }
  // Causal launches of at most two waves order their items pair-major over
  // all heads (every head's heaviest pairs first), so no group of heads
  // starts its heaviest items late; larger launches keep the kernel's
  // groups of 8 heads, whose CTAs share K/V in L2 (measured on B200: C3,
  // 256 items = 1.7 waves, 340 -> 417 TFLOPS with one group of all 32 heads;
  // C4, 6.9 waves, groups of 16 / 32 heads -1 % / -0.5 %, groups of 4 -5 %).
  // Key-split launches (under one wave) keep the groups (a 512-query chunk
  // of an 8k cache: 80.7 us with them, 82.0 us in one group).
  {
    const long long n_items = static_cast<long long>(k.n_qpairs) * B * k.heads * k.n_splits;
    p.head_group = (p.causal != 0 && k.n_splits == 1 && !k.dual && !k.decode &&
                    n_items <= 2LL * sm_count())
                       ? static_cast<int>(bh)
                       : fa::kFwdHeadGroup;
  }
  p.item0 = 0;
  p.item_end = 0;
  const bool use_ws = k.n_splits > 1 || k.dual;
  p.ws_o = use_ws ? static_cast<float*>(workspace) : nullptr;
  p.ws_lse = use_ws ? reinterpret_cast<float*>(static_cast<char*>(workspace) + k.ws_o_bytes)
                    : nullptr;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.debug_flags = g_debug_flags.load(std::memory_order_relaxed);
  p.trace = g_trace.load(std::memory_order_relaxed);
  p.epoch = g_epoch.fetch_add(1, std::memory_order_relaxed);
  p.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
  // Persistent shared-mode launches deal their last kDynRounds rounds from a
  // device-wide counter, so CTAs that drew lighter items take more of the
  // last ones (measured on B200: C5 causal +1.5 %, C5 +0.9 %; 1 or 4 dynamic
  // rounds gained less).
  constexpr int kDynRounds = 2;
  p.sched = 0;
  p.sched_round = 0;
  if (!k.decode && p.n_ctas > 0 && p.dual == 0 &&
      (p.debug_flags & FA_DEBUG_STATIC_DEAL) == 0) {
    const long long items = static_cast<long long>(k.n_qpairs) * B * k.heads * k.n_splits;
    const int rounds = static_cast<int>((items + p.n_ctas - 1) / p.n_ctas);
    if (rounds > kDynRounds) {
      p.sched = next_sched();
      p.sched_round = rounds - kDynRounds;
    }
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Wave tail: a non-causal pair-kernel launch of several waves whose last
  // wave is at most half full runs those last items on the tile kernel, as
  // twice as many one-tile items (each ~0.6 of a pair item's time), so the
  // last wave ends sooner.  (C5 sharded over 8 GPUs: 512 items, 3.46 waves.)
  // d = 128 only: at d = 64 the tile kernel runs a tile at more than 0.6 of
  // a pair item's time and the second launch costs more than it saves
  // (measured: C2, 192 items = 1.3 waves, 345 TFLOPS with the last 44 items
  // on the pair kernel against 331 with the split).
  const long long n_items = static_cast<long long>(k.n_qpairs) * B * k.heads * k.n_splits;
  const int sms = sm_count();
  const long long rem = n_items % sms;
  const bool tail = head_dim == 128 && !k.decode && !k.dual && !k.q_tile && !k.pair2 &&
                    k.n_splits == 1 &&
                    p.causal == 0 && n_items > sms && rem > 0 && 2 * rem <= sms &&
                    (g_debug_flags.load(std::memory_order_relaxed) & FA_DEBUG_NO_TAIL_SPLIT) == 0;
  cudaError_t e;
  if (tail) {
    const int full = static_cast<int>(n_items - rem);
    p.item_end = full;
    e = fa::launch_fwd(p, head_dim, bf16, s);
    if (e == cudaSuccess) {
      // pair items are head-major (item = bh * pairs + pair): the tiles of
      // items >= full are tile items >= bh * tiles + 2 * pair of item `full`
      fa::FwdParams pt = p;
      const int tiles = (k.rows + 127) / 128;
      pt.q_tile = 1;
      pt.n_qpairs = tiles;
      pt.item0 = (full / k.n_qpairs) * tiles + 2 * (full % k.n_qpairs);
      pt.item_end = 0;
      pt.n_ctas = 0;  // one CTA per tile item
      e = fa::launch_fwd(pt, head_dim, bf16, s);
    }
  } else {
    e = k.decode ? fa::launch_decode(p, head_dim, bf16, s) : fa::launch_fwd(p, head_dim, bf16, s);
  }
  if (e != cudaSuccess) return FA_ERR_LAUNCH;
  if (use_ws && fa::launch_combine(p, head_dim, bf16, s) != cudaSuccess) return FA_ERR_LAUNCH;
  return FA_OK;
}

// [T, H, d] packed rows viewed as 3-D (d, H, T) with a (64, 1, 128) box: one
// head's 128 consecutive tokens, laid out in shared memory exactly like a
// (64, 128, 1) box of make_map.  Rows >= T read as zeros.
bool make_map_packed(CUtensorMap* map, const void* base, int d, int h, long long t, bool bf16) {
  const MapKey key{base, t, h, d, 128, bf16 ? 1 : 0, 1};
  if (cached_map(map, key)) return true;
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(h),
                              static_cast<cuuint64_t>(t)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2,
                                 static_cast<cuuint64_t>(h) * static_cast<cuuint64_t>(d) * 2};
  const cuuint32_t box[3] = {64, 1, 128};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r =
      fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  remember_map(*map, key);
  return true;
}

// Launch of the attention kernel over per-batch row ranges (fa_fwd_varlen:
// packed = true; fa_fwd_padded: packed = false).  Nq / Nk are the largest
// sequence lengths (padded: the padded lengths); q_lim / k_lim bound the rows.
int launch_ranged(bool packed, const void* Q, const void* K, const void* V, void* O, float* lse,
                  const int* q_lo, const int* q_hi, const int* k_lo, const int* k_hi, int B,
                  int Hq, int Hkv, int Nq, int Nk, int q_lim, int k_lim, int head_dim,
                  float scale, int causal, int dtype, void* stream) {
  const bool bf16 = dtype == FA_DTYPE_BF16;
  fa::FwdParams p;
  const bool maps_ok =
      packed ? (make_map_packed(&p.tm_q, Q, head_dim, Hq, q_lim, bf16) &&
                make_map_packed(&p.tm_k, K, head_dim, Hkv, k_lim > 0 ? k_lim : 1, bf16) &&
                make_map_packed(&p.tm_v, V, head_dim, Hkv, k_lim > 0 ? k_lim : 1, bf16))
             : (make_map(&p.tm_q, Q, head_dim, Nq, static_cast<long long>(B) * Hq, bf16) &&
                make_map(&p.tm_k, K, head_dim, Nk, static_cast<long long>(B) * Hkv, bf16) &&
                make_map(&p.tm_v, V, head_dim, Nk, static_cast<long long>(B) * Hkv, bf16));
  if (!maps_ok) return FA_ERR_TENSOR_MAP;
  p.o = O;
  p.o_rs = packed ? Hq * head_dim : head_dim;
  p.lse = lse;
  p.ranges = packed ? 1 : 2;
  p.causal_br = causal == FA_CAUSAL_BOTTOM_RIGHT ? 1 : 0;
  p.q_lim = q_lim;
  p.k_lim = k_lim;
  p.q_lo = q_lo;
  p.q_hi = q_hi;
  p.k_lo = k_lo;
  p.k_hi = k_hi;
  p.B = B;
  p.heads = Hq;
  p.Hkv = Hkv;
  p.Nq = Nq;
  p.Nk = Nk;
  p.group = Hq / Hkv;
  p.q_tile = use_tile_kernel(static_cast<long long>((Nq + 255) / 256) * B * Hq) ? 1 : 0;
  p.n_qpairs = p.q_tile ? (Nq + 127) / 128 : (Nq + 255) / 256;
  p.n_kv_tiles = (Nk + 127) / 128;
  p.causal = causal != FA_CAUSAL_NONE ? 1 : 0;
  // packed: per-sequence offsets come from causal_br in the kernel; padded:
  // the rule of the full padded rows
  p.causal_off = (!packed && causal == FA_CAUSAL_BOTTOM_RIGHT) ? Nk - Nq : 0;
  p.pos_mod = 0x7fffffff;
  p.n_splits = 1;
  p.tiles_per_split = p.n_kv_tiles;
  p.dual = 0;
  p.n_ctas = 0;
  p.head_group = fa::kFwdHeadGroup;
  p.item0 = 0;
  p.item_end = 0;
  p.sched = 0;
  p.sched_round = 0;
  p.ws_o = nullptr;
  p.ws_lse = nullptr;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.debug_flags = g_debug_flags.load(std::memory_order_relaxed);
  p.trace = g_trace.load(std::memory_order_relaxed);
  p.epoch = g_epoch.fetch_add(1, std::memory_order_relaxed);
  p.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
  if (fa::launch_fwd(p, head_dim, bf16, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return FA_ERR_LAUNCH;
  return FA_OK;
}

}  // namespace

extern "C" {

int fa_fwd(const void* Q, const void* K, const void* V, void* O, float* lse, int B, int Hq,
           int Hkv, int N, int head_dim, float scale, int causal, int dtype, void* stream) {
  if (causal != 0 && causal != 1) return FA_ERR_INVALID_ARG;
  bool empty = false;
  if (int rc = check_args(Q, K, V, O, lse, B, Hq, Hkv, N, N, head_dim, scale, causal, dtype,
                          &empty))
    return rc;
  if (empty) return FA_OK;
  return launch_attention(Q, K, V, O, lse, B, Hq, Hkv, N, N, head_dim, scale, causal, dtype,
                          nullptr, 0, stream);
}

int fa_fwd_kvcache(const void* Q, const void* K, const void* V, void* O, float* lse, int B,
                   int Hq, int Hkv, int Nq, int Nk, int head_dim, float scale, int causal,
                   int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  bool empty = false;
  if (int rc = check_args(Q, K, V, O, lse, B, Hq, Hkv, Nq, Nk, head_dim, scale, causal, dtype,
                          &empty))
    return rc;
  if (empty) return FA_OK;
  return launch_attention(Q, K, V, O, lse, B, Hq, Hkv, Nq, Nk, head_dim, scale, causal, dtype,
                          workspace, workspace_bytes, stream);
}

size_t fa_bwd_workspace_bytes(int B, int Hq, int N) {
  if (B <= 0 || Hq <= 0 || N <= 0) return 0;
  const size_t n_pad = (static_cast<size_t>(N) + 127) / 128 * 128;
  // per query row: -LSE*log2(e) and -D (fp32); per 128-row query tile: two
  // 4 KB operand tiles (BwdParams::vt)
  return 2 * static_cast<size_t>(B) * Hq * n_pad * sizeof(float) +
         static_cast<size_t>(B) * Hq * (n_pad / 128) * 8192;
}

}  // extern "C"

namespace {

// fa_bwd, fa_bwd_padded and fa_bwd_varlen: ranges (q_lo, q_hi, k_lo, k_hi)
// all null or all set; cu (cu_seqlens of a packed batch, `total` rows, N the
// longest sequence) or null.
int launch_backward(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                    const float* lse, void* dQ, void* dK, void* dV, const int* q_lo,
                    const int* q_hi, const int* k_lo, const int* k_hi, const int* cu, int total,
                    int B, int Hq, int Hkv, int N, int head_dim, float scale, int causal,
                    int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (B < 0 || Hq < 0 || Hkv < 0 || N < 0) return FA_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_DTYPE;
  if (causal != 0 && causal != 1) return FA_ERR_INVALID_ARG;
  if (B == 0 || Hq == 0 || N == 0) return FA_OK;
  if (Hkv == 0) return FA_ERR_INVALID_ARG;
  if (Hq % Hkv != 0) return FA_ERR_GQA_DIVISIBILITY;
  if (!Q || !K || !V || !O || !dO || !lse || !dQ || !dK || !dV || !workspace)
    return FA_ERR_INVALID_ARG;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(dO) ||
      !aligned16(dQ) || !aligned16(dK) || !aligned16(dV) || !aligned16(workspace) ||
      (reinterpret_cast<uintptr_t>(lse) & 3u))
    return FA_ERR_ALIGNMENT;
  if (workspace_bytes < fa_bwd_workspace_bytes(B, Hq, N)) return FA_ERR_INVALID_ARG;
  if (!std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  const long long n_tiles = (static_cast<long long>(N) + 127) / 128;
  if (N > (1 << 30) || static_cast<long long>(B) * Hq * n_tiles > 0x7fffffffLL)
    return FA_ERR_TOO_LARGE;
  if (int rc = check_device()) return rc;

  fa::BwdParams p;
  const bool bf16 = dtype == FA_DTYPE_BF16;
  const long long bhq = static_cast<long long>(B) * Hq, bhk = static_cast<long long>(B) * Hkv;
  const bool maps_ok =
      cu ? (make_map_packed(&p.tm_q, Q, head_dim, Hq, total, bf16) &&
            make_map_packed(&p.tm_do, dO, head_dim, Hq, total, bf16) &&
            make_map_packed(&p.tm_k, K, head_dim, Hkv, total, bf16) &&
            make_map_packed(&p.tm_v, V, head_dim, Hkv, total, bf16))
         : (make_map(&p.tm_q, Q, head_dim, N, bhq, bf16) &&
            make_map(&p.tm_do, dO, head_dim, N, bhq, bf16) &&
            make_map(&p.tm_k, K, head_dim, N, bhk, bf16) &&
            make_map(&p.tm_v, V, head_dim, N, bhk, bf16));
  if (!maps_ok) return FA_ERR_TENSOR_MAP;
  p.dq = dQ;
  p.dk = dK;
  p.dv = dV;
  p.q_lo = q_lo;
  p.q_hi = q_hi;
  p.k_lo = k_lo;
  p.k_hi = k_hi;
  p.cu = cu;
  p.total = total;
  p.n_tiles = static_cast<int>(n_tiles);
  p.n_pad = p.n_tiles * 128;
  p.l2 = static_cast<const float*>(workspace);
  p.dd = static_cast<const float*>(workspace) + static_cast<size_t>(bhq) * p.n_pad;
  p.vt = static_cast<const uint8_t*>(workspace) + 2 * static_cast<size_t>(bhq) * p.n_pad * sizeof(float);
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.N = N;
  p.group = Hq / Hkv;
  p.causal = causal;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.trace = g_trace.load(std::memory_order_relaxed);
  p.epoch = g_epoch.fetch_add(1, std::memory_order_relaxed);
  p.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
  const cudaError_t e = fa::launch_bwd(p, O, dO, lse, head_dim, bf16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

}  // namespace

extern "C" {

int fa_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
           const float* lse, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv, int N,
           int head_dim, float scale, int causal, int dtype, void* workspace,
           size_t workspace_bytes, void* stream) {
  return launch_backward(Q, K, V, O, dO, lse, dQ, dK, dV, nullptr, nullptr, nullptr, nullptr,
                         nullptr, 0, B, Hq, Hkv, N, head_dim, scale, causal, dtype, workspace,
                         workspace_bytes, stream);
}

int fa_bwd_padded(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                  const float* lse, const int* q_start, const int* q_end, const int* k_start,
                  const int* k_end, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv, int N,
                  int head_dim, float scale, int causal, int dtype, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (B > 0 && Hq > 0 && N > 0 && (!q_start || !q_end || !k_start || !k_end))
    return FA_ERR_INVALID_ARG;
  return launch_backward(Q, K, V, O, dO, lse, dQ, dK, dV, q_start, q_end, k_start, k_end,
                         nullptr, 0, B, Hq, Hkv, N, head_dim, scale, causal, dtype, workspace,
                         workspace_bytes, stream);
}

int fa_bwd_varlen(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                  const float* lse, const int* cu_seqlens, void* dQ, void* dK, void* dV, int B,
                  int Hq, int Hkv, int total, int max_seqlen, int head_dim, float scale,
                  int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (total < 0 || max_seqlen < 0) return FA_ERR_INVALID_ARG;
  if (B > 0 && Hq > 0 && total > 0 && max_seqlen > 0 && !cu_seqlens) return FA_ERR_INVALID_ARG;
  if (static_cast<long long>(total) * Hq * head_dim > (1LL << 40) ||
      static_cast<long long>(total) * Hkv * head_dim > (1LL << 40))
    return FA_ERR_TOO_LARGE;
  if (total == 0) return (B < 0 || Hq < 0 || Hkv < 0) ? FA_ERR_INVALID_ARG : FA_OK;
  return launch_backward(Q, K, V, O, dO, lse, dQ, dK, dV, nullptr, nullptr, nullptr, nullptr,
                         cu_seqlens, total, B, Hq, Hkv, max_seqlen, head_dim, scale, causal, dtype,
                         workspace, workspace_bytes, stream);
}

int fa_fwd_varlen(const void* Q, const void* K, const void* V, void* O, float* lse,
                  const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                  int total_q, int total_k, int max_seqlen_q, int max_seqlen_k, int head_dim,
                  float scale, int causal, int dtype, void* stream) {
  if (total_q < 0 || total_k < 0 || max_seqlen_q < 0 || max_seqlen_k < 0)
    return FA_ERR_INVALID_ARG;
  bool empty = false;
  // the shape checks of a [B, Hq, max_seqlen_q, d] call; rows then come from
  // the offsets
  if (int rc = check_args(Q, K, V, O, lse, B, Hq, Hkv, max_seqlen_q, max_seqlen_k > 0 ? max_seqlen_k : 1,
                          head_dim, scale, causal, dtype, &empty))
    return rc;
  if (empty || total_q == 0) return FA_OK;
  if (!cu_seqlens_q || !cu_seqlens_k) return FA_ERR_INVALID_ARG;
  if (static_cast<long long>(total_q) * Hq * head_dim > (1LL << 40) ||
      static_cast<long long>(total_k) * Hkv * head_dim > (1LL << 40))
    return FA_ERR_TOO_LARGE;
  // total_k = 0: every key range clamps to empty, so every row gets O = 0 and
  // LSE = -inf and K/V are never read (their maps still need one row)
  return launch_ranged(true, Q, K, V, O, lse, cu_seqlens_q, cu_seqlens_q + 1, cu_seqlens_k,
                       cu_seqlens_k + 1, B, Hq, Hkv, max_seqlen_q,
                       max_seqlen_k > 0 ? max_seqlen_k : 1, total_q, total_k, head_dim, scale,
                       causal, dtype, stream);
}

int fa_fwd_padded(const void* Q, const void* K, const void* V, void* O, float* lse,
                  const int* q_start, const int* q_end, const int* k_start, const int* k_end,
                  int B, int Hq, int Hkv, int Nq, int Nk, int head_dim, float scale, int causal,
                  int dtype, void* stream) {
  bool empty = false;
  if (int rc = check_args(Q, K, V, O, lse, B, Hq, Hkv, Nq, Nk, head_dim, scale, causal, dtype,
                          &empty))
    return rc;
  if (empty) return FA_OK;
  if (!q_start || !q_end || !k_start || !k_end) return FA_ERR_INVALID_ARG;
  return launch_ranged(false, Q, K, V, O, lse, q_start, q_end, k_start, k_end, B, Hq, Hkv, Nq,
                       Nk, Nq, Nk, head_dim, scale, causal, dtype, stream);
}

size_t fa_fwd_kvcache_workspace_bytes(int B, int Hq, int Hkv, int Nq, int Nk, int head_dim) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Nq <= 0 || Nk <= 0 || Hq % Hkv != 0 ||
      (head_dim != 64 && head_dim != 128))
    return 0;
  return make_plan(B, Hq, Hkv, Nq, Nk, head_dim, true).ws_bytes;
}

static void legacy_fwd(const char* tag, const void* Q, const void* K, const void* V, void* O,
                       int batch, int heads, int seq_len, int head_dim, float scale, bool causal) {
  const int rc = fa_fwd(Q, K, V, O, nullptr, batch, heads, heads, seq_len, head_dim, scale,
                        causal ? 1 : 0, FA_DTYPE_F16, nullptr);
  if (rc != FA_OK) {
    if (rc == FA_ERR_UNSUPPORTED_HEAD_DIM)
      fprintf(stderr, "[%s] head_dim=%d not supported\n", tag, head_dim);
    else
      fprintf(stderr, "[%s] %s\n", tag, fa_error_string(rc));
    return;
  }
  cudaDeviceSynchronize();
}

void launch_flash_attention_forward(const void* Q, const void* K, const void* V, void* O,
                                    int batch, int heads, int seq_len, int head_dim, float scale,
                                    bool causal) {
  legacy_fwd("flash_attn", Q, K, V, O, batch, heads, seq_len, head_dim, scale, causal);
}

void launch_flash_attention_forward_scalar(const void* Q, const void* K, const void* V, void* O,
                                           int batch, int heads, int seq_len, int head_dim,
                                           float scale, bool causal) {
  if (head_dim != 64) {
    fprintf(stderr, "[flash_attn_scalar] head_dim=%d not supported\n", head_dim);
    return;
  }
  legacy_fwd("flash_attn_scalar", Q, K, V, O, batch, heads, seq_len, head_dim, scale, causal);
}

void launch_flash_attention_forward_wmma_qk(const void* Q, const void* K, const void* V, void* O,
                                            int batch, int heads, int seq_len, int head_dim,
                                            float scale, bool causal) {
  if (head_dim != 64) {
    fprintf(stderr, "[flash_attn_wmma_qk] head_dim=%d not supported\n", head_dim);
    return;
  }
  legacy_fwd("flash_attn_wmma_qk", Q, K, V, O, batch, heads, seq_len, head_dim, scale, causal);
}

int fa_naive_fwd(const void* Q, const void* K, const void* V, void* O, int batch, int heads,
                 int seq_len, int head_dim, float scale, int causal, float* workspace,
                 void* stream) {
  if (batch < 0 || heads < 0 || seq_len < 0 || head_dim <= 0) return FA_ERR_INVALID_ARG;
  if (batch == 0 || heads == 0 || seq_len == 0) return FA_OK;
  if (!Q || !K || !V || !O || !workspace) return FA_ERR_INVALID_ARG;
  const long long bh = static_cast<long long>(batch) * heads;
  if (bh > 65535) return FA_ERR_TOO_LARGE;  // grid.z limit
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* q = static_cast<const __half*>(Q);
  const __half* k = static_cast<const __half*>(K);
  const __half* v = static_cast<const __half*>(V);
  {
    dim3 block(32, 8);
    dim3 grid((seq_len + 31) / 32, (seq_len + 7) / 8, static_cast<unsigned>(bh));
    naive_qk_kernel<<<grid, block, 0, s>>>(q, k, workspace, seq_len, head_dim, scale, causal);
  }
  {
    dim3 block(256);
    dim3 grid((seq_len + 7) / 8, static_cast<unsigned>(bh));
    naive_softmax_kernel<<<grid, block, 0, s>>>(workspace, seq_len);
  }
  {
    dim3 block(32, 8);
    dim3 grid((head_dim + 31) / 32, (seq_len + 7) / 8, static_cast<unsigned>(bh));
    naive_pv_kernel<<<grid, block, 0, s>>>(workspace, v, static_cast<__half*>(O), seq_len,
                                           head_dim);
  }
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

void launch_naive_attention(const void* Q, const void* K, const void* V, void* O, int batch,
                            int heads, int seq_len, int head_dim, float scale, bool causal,
                            float* workspace) {
  const int rc = fa_naive_fwd(Q, K, V, O, batch, heads, seq_len, head_dim, scale, causal ? 1 : 0,
                              workspace, nullptr);
  if (rc != FA_OK) fprintf(stderr, "[naive_attention] %s\n", fa_error_string(rc));
  cudaDeviceSynchronize();
}

int flatargs_launch(const void* Q, const void* K, const void* V, void* O, int B, int H, int N,
                    float scale, void* stream) {
  return fa_fwd(Q, K, V, O, nullptr, B, H, H, N, 64, scale, 0, FA_DTYPE_F16, stream);
}

int launch_v2(const void* Q, const void* K, const void* V, void* O, int B, int H, int N,
              float scale, int mode, void* stream) {
  if (mode != 0 && mode != 1) return FA_ERR_INVALID_ARG;
  return fa_fwd(Q, K, V, O, nullptr, B, H, H, N, 64, scale, mode, FA_DTYPE_F16, stream);
}

int fa_device_status(int reset) {
  unsigned long long st = 0;
  if (fa::read_status(&st, reset != 0) != cudaSuccess) return FA_ERR_CUDA;
  return static_cast<int>(st & 0xffffffffull);
}

void fa_set_watchdog_ns(unsigned long long ns) { g_timeout_ns.store(ns ? ns : 1ull); }

void fa_set_debug_flags(int flags) { g_debug_flags.store(flags); }

// Development hook: device buffer for FA_TRACE builds (8*64*32 int64), or NULL.
void fa_set_trace_buffer(void* buf) { g_trace.store(static_cast<long long*>(buf)); }

const char* fa_error_string(int code) {
  switch (code) {
    case FA_OK: return "ok";
    case FA_ERR_INVALID_ARG: return "invalid argument";
    case FA_ERR_UNSUPPORTED_HEAD_DIM: return "supports head_dim=64 or 128 only";
    case FA_ERR_GQA_DIVISIBILITY: return "Q heads not divisible by K/V heads";
    case FA_ERR_ALIGNMENT: return "Q/K/V/O must be 16-byte aligned (LSE 4-byte)";
    case FA_ERR_DTYPE: return "dtype must be FA_DTYPE_F16 or FA_DTYPE_BF16";
    case FA_ERR_TENSOR_MAP: return "TMA descriptor creation failed";
    case FA_ERR_LAUNCH: return "kernel launch failed";
    case FA_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case FA_ERR_CUDA: return "CUDA runtime call failed";
    case FA_ERR_TOO_LARGE: return "problem size exceeds the kernel's index range";
    case FA_ERR_SCRATCH_LIMIT:
      return "batch*heads*seq_len^2 exceeds the 4Mi-float scratch of fa_naive_fwd_noalloc";
    default: break;
  }
  if (code >= FA_ERR_TIMEOUT_BASE) return "device watchdog: an in-kernel wait timed out";
  return "unknown error";
}

int fa_smem_bytes(int head_dim) {
  if (head_dim != 64 && head_dim != 128) return -1;
  return fa::smem_bytes_for(head_dim);
}

const char* fa_version(void) { return "fa_b200 0.1.0 (sm_100a tcgen05)"; }

}  // extern "C"

// ------------------------------------------------------------------ no-alloc
// Materialised attention for callers that must not allocate device memory
// while they run (hosts whose allocator is closed after start-up, real-time
// or embedded loops, runtimes that own all device memory): the score matrix
// lives in a fixed file-scope device array instead of a caller-provided or
// freshly allocated workspace.  The array is part of this library's device
// image, so every GPU that loads the library keeps these 16 MiB until the
// process exits.
namespace {

constexpr unsigned long long kNoAllocScratchFloats = 4ull << 20;  // 16 MiB of fp32 scores
__device__ __align__(256) float g_naive_noalloc_scratch[kNoAllocScratchFloats];

// Device address of the scratch array for the current device.  Host code may
// not pass the symbol itself to a kernel (on the host it names a host-side
// stand-in); the address is looked up on every call, with the calling
// thread's current device, so it stays valid after a cudaDeviceReset reloads
// this module.  The lookup allocates nothing.
int noalloc_scratch(float** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_naive_noalloc_scratch) != cudaSuccess || p == nullptr)
    return FA_ERR_CUDA;
  *out = static_cast<float*>(p);
  return FA_OK;
}

}  // namespace

extern "C" int fa_naive_fwd_noalloc(const void* Q, const void* K, const void* V, void* O,
                                    int batch, int heads, int seq_len, int head_dim, float scale,
                                    int causal, void* stream) {
  if (batch < 0 || heads < 0 || seq_len < 0 || head_dim <= 0) return FA_ERR_INVALID_ARG;
  if (batch == 0 || heads == 0 || seq_len == 0) return FA_OK;
  const unsigned long long need = static_cast<unsigned long long>(batch) * heads *
                                  static_cast<unsigned long long>(seq_len) * seq_len;
  if (need > kNoAllocScratchFloats) return FA_ERR_SCRATCH_LIMIT;
  float* ws = nullptr;
  if (int rc = noalloc_scratch(&ws)) return rc;
  // Every score the softmax and PV kernels read is written by the QK^T kernel
  // of the same call first, so the shared array needs no clearing.
  return fa_naive_fwd(Q, K, V, O, batch, heads, seq_len, head_dim, scale, causal, ws, stream);
}
