// Shared host code of the standalone CLIs (flash_mha_flatargs, flash_mha_v2).
//
// Same command line and stdout contract as the reference tools
// (flash-attention-sm75-fused/src/flash_mha_flatargs.cu:652-691,
//  flash-attention-sm75-fused/src/flash_mha_v2.cu:790-816):
//   ./tool                 -> small validated cases + a sweep table
//   ./tool B H N [outer [inner]]
// Timing: 3 warm-up launches, `outer` rounds of `inner` back-to-back launches
// timed with CUDA events; min / median / max of the per-launch times.
// Validation (when B*H*N*N*64 < 3e8): inputs uniform(-0.25, 0.25) from
// std::srand(42), fp32 CPU reference, pass if max |err| < 5e-2.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "fa_b200.h"

namespace cli {

constexpr int kD = 64;

inline void check(cudaError_t e, const char* where) {
  if (e != cudaSuccess) {
    std::fprintf(stderr, "CUDA error in %s: %s\n", where, cudaGetErrorString(e));
    std::exit(1);
  }
}

inline void check_fa(int rc, const char* where) {
  if (rc != FA_OK) {
    std::fprintf(stderr, "fa error in %s: %s\n", where, fa_error_string(rc));
    std::exit(1);
  }
}

inline float rand_val() { return (std::rand() / (float)RAND_MAX - 0.5f) * 0.5f; }

// fp32 CPU attention over fp16 inputs, [B, H, N, d]; causal = top-left.
inline void cpu_attention(const std::vector<__half>& Q, const std::vector<__half>& K,
                          const std::vector<__half>& V, std::vector<float>& O, int B, int H,
                          int N, int d, float scale, bool causal) {
  std::vector<float> s(N);
  for (int bh = 0; bh < B * H; ++bh) {
    const size_t off = (size_t)bh * N * d;
    for (int i = 0; i < N; ++i) {
      const int kmax = causal ? i + 1 : N;
      float mx = -FLT_MAX;
      for (int j = 0; j < kmax; ++j) {
        float acc = 0.f;
        for (int c = 0; c < d; ++c)
          acc += __half2float(Q[off + (size_t)i * d + c]) * __half2float(K[off + (size_t)j * d + c]);
        s[j] = acc * scale;
        mx = std::max(mx, s[j]);
      }
      float sum = 0.f;
      for (int j = 0; j < kmax; ++j) {
        s[j] = std::exp(s[j] - mx);
        sum += s[j];
      }
      for (int c = 0; c < d; ++c) {
        float acc = 0.f;
        for (int j = 0; j < kmax; ++j) acc += s[j] * __half2float(V[off + (size_t)j * d + c]);
        O[off + (size_t)i * d + c] = acc / sum;
      }
    }
  }
}

inline bool validate(const std::vector<__half>& out, const std::vector<float>& ref, int B, int H,
                     int N, int d, const char* label, float tol = 5e-2f) {
  float max_abs = 0.f, max_rel = 0.f;
  int wb = 0, wh = 0, wr = 0, wc = 0;
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
      for (int i = 0; i < N; ++i)
        for (int c = 0; c < d; ++c) {
          const size_t k = (((size_t)b * H + h) * N + i) * d + c;
          const float g = __half2float(out[k]);
          const float err = std::fabs(g - ref[k]);
          if (err > max_abs) {
            max_abs = err;
            max_rel = std::fabs(ref[k]) > 1e-6f ? err / std::fabs(ref[k]) : err;
            wb = b, wh = h, wr = i, wc = c;
          }
        }
  const bool ok = max_abs < tol;
  std::printf("  [%s] max_abs=%.6f  max_rel=%.4f%%  at[b=%d h=%d r=%d c=%d]  %s\n", label, max_abs,
              max_rel * 100.f, wb, wh, wr, wc, ok ? "PASS" : "FAIL");
  return ok;
}

struct Stats {
  double min_ms, med_ms, max_ms;
};

// `launch` enqueues one forward on the legacy default stream.
template <class F>
Stats bench(F launch, int outer, int inner) {
  for (int i = 0; i < 3; ++i) launch();
  check(cudaDeviceSynchronize(), "warm-up");
  outer = std::max(1, std::min(outer, 64));
  inner = std::max(1, inner);
  std::vector<float> t(outer);
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  for (int r = 0; r < outer; ++r) {
    cudaEventRecord(a);
    for (int i = 0; i < inner; ++i) launch();
    cudaEventRecord(b);
    cudaEventSynchronize(b);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    t[r] = ms / inner;
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  std::sort(t.begin(), t.end());
  return {t.front(), t[outer / 2], t.back()};
}

struct Buffers {
  __half *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
  size_t n = 0;
  explicit Buffers(size_t elems) : n(elems) {
    check(cudaMalloc(&q, n * sizeof(__half)), "malloc Q");
    check(cudaMalloc(&k, n * sizeof(__half)), "malloc K");
    check(cudaMalloc(&v, n * sizeof(__half)), "malloc V");
    check(cudaMalloc(&o, n * sizeof(__half)), "malloc O");
  }
  ~Buffers() {
    cudaFree(q);
    cudaFree(k);
    cudaFree(v);
    cudaFree(o);
  }
};

// Host inputs from std::srand(42); large benchmark-only cases fill the device
// buffers with the same generator instead of zeros.
inline void fill_inputs(Buffers& buf, std::vector<__half>& hq, std::vector<__half>& hk,
                        std::vector<__half>& hv) {
  hq.resize(buf.n);
  hk.resize(buf.n);
  hv.resize(buf.n);
  std::srand(42);
  for (size_t i = 0; i < buf.n; ++i) {
    hq[i] = __float2half(rand_val());
    hk[i] = __float2half(rand_val());
    hv[i] = __float2half(rand_val());
  }
  check(cudaMemcpy(buf.q, hq.data(), buf.n * sizeof(__half), cudaMemcpyHostToDevice), "H2D Q");
  check(cudaMemcpy(buf.k, hk.data(), buf.n * sizeof(__half), cudaMemcpyHostToDevice), "H2D K");
  check(cudaMemcpy(buf.v, hv.data(), buf.n * sizeof(__half), cudaMemcpyHostToDevice), "H2D V");
}

inline void print_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceProp prop;
  check(cudaGetDeviceProperties(&prop, dev), "device properties");
  std::printf("Device: %s  SM%d%d  %d SMs\n", prop.name, prop.major, prop.minor,
              prop.multiProcessorCount);
}

}  // namespace cli
