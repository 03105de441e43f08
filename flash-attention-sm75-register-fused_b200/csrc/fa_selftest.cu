// Stage tests of the attention kernel's building blocks, built as a separate
// test library (lib/libfa_selftest.so) that only tests/ load:
//
//   fa_selftest_exp2     the FMA-pipe polynomial exp2 (exp2_poly2) and MUFU
//                        ex2.approx beside CUDA's exp2f, on given inputs
//   fa_selftest_softmax  the register softmax stage of one 128-key tile per
//                        row (row max, exp2(s*scale_log2 - m) with the
//                        kernel's MUFU / polynomial split, row sum, f16/bf16
//                        packing), from the same device code the kernel runs
//   fa_selftest_mma      one 128-row tile through TMA (128-byte swizzle), the
//                        shared-memory / instruction descriptors and tcgen05:
//                        S = A.B^T with both operands in shared memory (the
//                        kernel's Q.K^T), or O = P.V with P stored to tensor
//                        memory and V read MN-major (the kernel's P.V); the
//                        accumulator read back with tcgen05.ld
//
// These restate, for the B200 kernel, what the reference checks with its
// softmax known-answer test and layout probes
// (flash-attention-sm75-fused/src/test_warp_softmax.cu:144-241,
// probe_layout.cu).  Every wait is bounded; a wait that runs out records a
// status the host returns as an error.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "fa_softmax.cuh"
#include "sm100_ptx.cuh"

namespace {

using namespace fa;

__device__ int g_selftest_status = 0;

constexpr unsigned long long kTimeoutNs = 1000000000ull;  // 1 s per wait

__device__ bool wait_bounded(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = ptx::global_timer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::global_timer_ns() - t0 > kTimeoutNs) {
      atomicExch(&g_selftest_status, 1);
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------------ exp2
__global__ void selftest_exp2_kernel(const float* t, float* y_poly, float* y_mufu, float* y_ref,
                                     int n_pairs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_pairs) return;
  const float t0 = t[2 * i], t1 = t[2 * i + 1];
  float p0, p1;
  ptx::exp2_poly2(p0, p1, t0, t1);
  y_poly[2 * i] = p0;
  y_poly[2 * i + 1] = p1;
  y_mufu[2 * i] = ptx::ex2_approx(t0);
  y_mufu[2 * i + 1] = ptx::ex2_approx(t1);
  y_ref[2 * i] = exp2f(t0);
  y_ref[2 * i + 1] = exp2f(t1);
}

// ------------------------------------------------------------------ softmax
// One thread per row of 128 scores, the forward kernel's tile stage:
// unmasked rows (lim >= 128) reduce the raw scores and scale the maximum
// (sl >= 0), then exp2 with the polynomial on one pair in kEmuPeriod;
// masked rows (lim < 128: keys >= lim excluded) are pre-scaled, -inf past
// lim, all exponentials on MUFU.  Outputs: the scaled row max m, P in fp32
// and packed to f16/bf16 pairs, and the fp32 row sum.
template <bool BF16>
__global__ void selftest_softmax_kernel(const float* s, const int* lim, int rows, float sl,
                                        float* m_out, float* p_out, uint32_t* p16_out,
                                        float* sum_out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float x[128];
#pragma unroll
  for (int c = 0; c < 128; ++c) x[c] = s[static_cast<size_t>(r) * 128 + c];
  const int l = lim[r];
  const bool masked = l < 128;
  float m, sl_eff = sl;
  if (masked) {
#pragma unroll
    for (int c = 0; c < 128; c += 2) ptx::fmul2(x[c], x[c + 1], x[c], x[c + 1], sl, sl);
#pragma unroll
    for (int c = 0; c < 128; ++c)
      if (c >= l) x[c] = -INFINITY;
    m = row_extreme<128, false>(x);
    sl_eff = 1.0f;
  } else {
    m = row_extreme<128, false>(x) * sl;
  }
  const float neg_m = (m == -INFINITY) ? 0.f : -m;
  float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
#pragma unroll
  for (int h = 0; h < 4; ++h) {
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const int i = 32 * h + 2 * c;
      float e0, e1;
      if (masked)
        exp2_pair<false>(c, x[i], x[i + 1], sl_eff, neg_m, e0, e1);
      else
        exp2_pair<true>(c, x[i], x[i + 1], sl_eff, neg_m, e0, e1);
      if (c & 1)
        ptx::fadd2(b0, b1, b0, b1, e0, e1);
      else
        ptx::fadd2(a0, a1, a0, a1, e0, e1);
      p_out[static_cast<size_t>(r) * 128 + i] = e0;
      p_out[static_cast<size_t>(r) * 128 + i + 1] = e1;
      uint32_t pk;
      if constexpr (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(e0, e1);
        pk = *reinterpret_cast<uint32_t*>(&v);
      } else {
        __half2 v = __floats2half2_rn(e0, e1);
        pk = *reinterpret_cast<uint32_t*>(&v);
      }
      p16_out[static_cast<size_t>(r) * 64 + i / 2] = pk;
    }
  }
  ptx::fadd2(a0, a1, a0, a1, b0, b1);
  m_out[r] = m;
  sum_out[r] = a0 + a1;
}

// ------------------------------------------------------------------ mma
struct MmaTestParams {
  CUtensorMap tm_a;  // mode 0: A [128, d] K-major
  CUtensorMap tm_b;  // mode 0: B [128, d] K-major; mode 1: V [128 keys, d] (MN-major operand)
  const uint16_t* p;  // mode 1: P [128, 128] f16/bf16 rows (stored to tensor memory)
  float* out;         // mode 0: [128, 128]; mode 1: [128, d] fp32
  int mode, d;
};

constexpr int kTileBytes = 128 * 128 * 2;  // largest tile: 128 rows x d=128, 16-bit
constexpr int kBlockBytes = 128 * 128;     // one 64-column (128-byte) block of 128 rows
constexpr int kSmemBytes = 2 * kTileBytes + 64 + 1024;

template <bool BF16>
__global__ void __launch_bounds__(128, 1) selftest_mma_kernel(const __grid_constant__ MmaTestParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sA = ptx::smem_u32(smem);
  const uint32_t sB = sA + kTileBytes;
  const uint32_t bar_tma = sB + kTileBytes;
  const uint32_t bar_mma = bar_tma + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 2 * kTileBytes + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = p.d / 64;  // 64-column blocks of a d-wide tile

  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_tma, 1);
    ptx::mbar_init(bar_mma, 1);
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), 256);
    ptx::tmem_relinquish();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;

  if (p.mode == 1) {
    // P row r (thread r = TMEM lane r) as 64 packed pairs in columns 128..191
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.p) + threadIdx.x * 64;
    uint32_t v[32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = src[32 * h + i];
      ptx::tmem_st32(tmem + lane_off + 128 + 32 * h, v);
    }
    ptx::tmem_wait_st();
    ptx::tc_fence_before();
  }
  __syncthreads();
  ptx::tc_fence_after();

  bool ok = true;
  if (warp == 0) {
    if (ptx::elect_one()) {
      const uint32_t bytes = (p.mode == 0 ? 2u : 1u) * 128u * p.d * 2u;
      ptx::mbar_arrive_expect_tx(bar_tma, bytes);
      const uint64_t pol = ptx::policy_evict_first();
      for (int c = 0; c < cb; ++c) {
        if (p.mode == 0) ptx::tma_load_3d(sA + c * kBlockBytes, &p.tm_a, bar_tma, c * 64, 0, 0, pol);
        ptx::tma_load_3d(sB + c * kBlockBytes, &p.tm_b, bar_tma, c * 64, 0, 0, pol);
      }
    }
    __syncwarp();
    ok = __all_sync(0xffffffffu, wait_bounded(bar_tma, 0));
    if (ok) {
      ptx::tc_fence_after();
      const uint32_t fmt = BF16 ? 1u : 0u;
      if (ptx::elect_one()) {
        if (p.mode == 0) {
          // the forward kernel's S = Q K^T: K-major A and B, 16 keys of d per step
          const uint32_t idesc = ptx::make_idesc_f16(128, 128, fmt, 0, 0);
          const uint64_t ad = ptx::smem_desc_sw128(sA, 16, 1024);
          const uint64_t bd = ptx::smem_desc_sw128(sB, 16, 1024);
          for (int kk = 0; kk < p.d / 16; ++kk) {
            const uint64_t off = static_cast<uint64_t>(((kk / 4) * kBlockBytes + (kk % 4) * 32) >> 4);
            ptx::mma_ss(tmem, ad + off, bd + off, idesc, kk > 0 ? 1u : 0u);
          }
        } else {
          // the forward kernel's O = P V: P from TMEM, V MN-major, 16 keys per step
          const uint32_t idesc = ptx::make_idesc_f16(128, p.d, fmt, 0, 1);
          const uint64_t vd = ptx::smem_desc_sw128(sB, kBlockBytes, 1024);
          for (int kk = 0; kk < 8; ++kk)
            ptx::mma_ts(tmem, tmem + 128 + kk * 8, vd + static_cast<uint64_t>((kk * 2048) >> 4),
                        idesc, kk > 0 ? 1u : 0u);
        }
        ptx::mma_commit(bar_mma);
      }
      __syncwarp();
    }
  }
  // every thread learns whether warp 0 issued the products
  ok = __syncthreads_and(ok ? 1 : 0) != 0;
  if (ok && wait_bounded(bar_mma, 0)) {
    ptx::tc_fence_after();
    const int ncols = p.mode == 0 ? 128 : p.d;
    for (int c0 = 0; c0 < ncols; c0 += 32) {
      uint32_t v[32];
      ptx::tmem_ld32(tmem + lane_off + c0, v);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i)
        p.out[static_cast<size_t>(warp * 32 + lane) * ncols + c0 + i] = __uint_as_float(v[i]);
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 256);
  }
}

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

// [128, d] 16-bit rows as the forward kernel describes a head: (d, 128, 1),
// box (64, 128, 1), 128-byte swizzle.
bool tile_map(CUtensorMap* map, const void* base, int d, bool bf16) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), 128, 1};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2,
                                 static_cast<cuuint64_t>(d) * 2 * 128};
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int finish(cudaStream_t s) {
  if (cudaGetLastError() != cudaSuccess) return 2;
  if (cudaStreamSynchronize(s) != cudaSuccess) return 3;
  int st = 0;
  if (cudaMemcpyFromSymbol(&st, g_selftest_status, sizeof(st)) != cudaSuccess) return 3;
  if (st != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_selftest_status, &zero, sizeof(zero));
    return 4;  // a bounded wait ran out
  }
  return 0;
}

}  // namespace

extern "C" {

// y_poly / y_mufu / y_ref[i] = exp2_poly2 / ex2.approx / exp2f of t[i];
// n even.  Device pointers; synchronous.  Returns 0 or an error code.
int fa_selftest_exp2(const float* t, float* y_poly, float* y_mufu, float* y_ref, int n,
                     void* stream) {
  if (n <= 0 || (n & 1)) return 1;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int pairs = n / 2;
  selftest_exp2_kernel<<<(pairs + 255) / 256, 256, 0, s>>>(t, y_poly, y_mufu, y_ref, pairs);
  return finish(s);
}

// The forward kernel's softmax stage on `rows` rows of 128 fp32 scores:
// lim[r] < 128 masks keys >= lim[r] (the diagonal-tile path).  Outputs
// m [rows], p [rows, 128] fp32, p16 [rows, 64] packed pairs, sum [rows].
int fa_selftest_softmax(const float* s, const int* lim, int rows, float scale_log2, int bf16,
                        float* m, float* p, uint32_t* p16, float* sum, void* stream) {
  if (rows <= 0 || !(scale_log2 >= 0.f)) return 1;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (bf16)
    selftest_softmax_kernel<true><<<(rows + 63) / 64, 64, 0, st>>>(s, lim, rows, scale_log2, m, p,
                                                                   p16, sum);
  else
    selftest_softmax_kernel<false><<<(rows + 63) / 64, 64, 0, st>>>(s, lim, rows, scale_log2, m,
                                                                    p, p16, sum);
  return finish(st);
}

// One tcgen05 tile.  mode 0: out[128,128] = A[128,d] . B[128,d]^T; mode 1:
// out[128,d] = P[128,128] . V[128,d] with P (passed as `a`) stored to tensor
// memory.  16-bit inputs (bf16 != 0: bfloat16), d in {64, 128}, 16-byte
// aligned device pointers.  Synchronous.  Returns 0 or an error code.
int fa_selftest_mma(const void* a, const void* b, float* out, int mode, int d, int bf16,
                    void* stream) {
  if ((mode != 0 && mode != 1) || (d != 64 && d != 128)) return 1;
  MmaTestParams p{};
  if (mode == 0 && !tile_map(&p.tm_a, a, d, bf16 != 0)) return 5;
  if (!tile_map(&p.tm_b, b, d, bf16 != 0)) return 5;
  p.p = static_cast<const uint16_t*>(a);
  p.out = out;
  p.mode = mode;
  p.d = d;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto kern = bf16 ? selftest_mma_kernel<true> : selftest_mma_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess)
    return 2;
  kern<<<1, 128, kSmemBytes, s>>>(p);
  return finish(s);
}

}  // extern "C"
