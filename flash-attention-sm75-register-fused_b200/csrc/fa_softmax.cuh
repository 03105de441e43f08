// Register-softmax building blocks of the attention forward, shared by the
// kernel (fa_fwd_sm100.cu) and the stage tests (fa_selftest.cu): the
// three-input row max, and exp2(s * scale_log2 - m) for a pair of scores with
// a fixed fraction of the pairs on the FMA-pipe polynomial instead of MUFU.
//
// Counterpart of the reference's register softmax
// (flash-attention-sm75-fused/include/warp_softmax.cuh:38-118: row max,
// exp(s - m), row sum), here one query row per thread over a 128-key tile.
#pragma once
#include <cstdint>

#include "sm100_ptx.cuh"

namespace fa {

// Fraction of exponentials evaluated by the FMA-pipe polynomial instead of
// the MUFU unit: pair c of every group of kEmuPeriod pairs uses the
// polynomial when c % kEmuPeriod >= kEmuPeriod - kEmuCount.
#ifndef FA_EMU_PERIOD
#define FA_EMU_PERIOD 4
#endif
#ifndef FA_EMU_COUNT
#define FA_EMU_COUNT 1
#endif
constexpr int kEmuPeriod = FA_EMU_PERIOD;
constexpr int kEmuCount = FA_EMU_COUNT;

// Three-input max / min (sm_100 forms of max.f32 / min.f32).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Max (kMin: min) of N scores in four independent three-input chains.
template <int N, bool kMin>
__device__ __forceinline__ float row_extreme(const float (&x)[N]) {
  static_assert(N % 8 == 0 && N >= 16, "row length");
  auto op3 = [](float a, float b, float c) { return kMin ? fmin3(a, b, c) : fmax3(a, b, c); };
  float a = x[0], b = x[1], c = x[2], d = x[3];
#pragma unroll
  for (int i = 4; i + 8 <= N; i += 8) {
    a = op3(a, x[i], x[i + 1]);
    b = op3(b, x[i + 2], x[i + 3]);
    c = op3(c, x[i + 4], x[i + 5]);
    d = op3(d, x[i + 6], x[i + 7]);
  }
  a = op3(a, x[N - 4], x[N - 3]);
  b = op3(b, x[N - 2], x[N - 1]);
  return op3(a, b, kMin ? fminf(c, d) : fmaxf(c, d));
}

// (e0, e1) = exp2(x0 * sl - m), exp2(x1 * sl - m) for pair c of a 16-pair
// quarter (neg_m = -m): one packed FMA, then MUFU ex2 or, for the pairs the
// emulation pattern selects (kEmulate), the degree-3 polynomial.
// kPeriod overrides the period of the pattern (the count stays kEmuCount).
template <bool kEmulate, int kPeriod = kEmuPeriod>
__device__ __forceinline__ void exp2_pair(int c, float x0, float x1, float sl, float neg_m,
                                          float& e0, float& e1) {
  static_assert(kPeriod > kEmuCount, "emulation pattern");
  float t0, t1;
  ptx::ffma2(t0, t1, x0, x1, sl, sl, neg_m, neg_m);
  if (kEmulate && (c % kPeriod) >= kPeriod - kEmuCount) {
    ptx::exp2_poly2(e0, e1, t0, t1);
  } else {
    e0 = ptx::ex2_approx(t0);
    e1 = ptx::ex2_approx(t1);
  }
}

}  // namespace fa
