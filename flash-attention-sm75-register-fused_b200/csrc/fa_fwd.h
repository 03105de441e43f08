// Internal interface between the host C-ABI (fa_abi.cu) and the sm_100a
// kernel (fa_fwd_sm100.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "fa_b200.h"

namespace fa {

// Kernel parameters; passed by value as a __grid_constant__ so the TMA
// descriptors live in parameter space.
struct alignas(64) FwdParams {
  CUtensorMap tm_q;  // 3-D (d, N, B*Hq),  box (64, 128, 1), 128-byte swizzle
  CUtensorMap tm_k;  // 3-D (d, N, B*Hkv)
  CUtensorMap tm_v;  // 3-D (d, N, B*Hkv)
  void* o;           // [B, Hq, N, d] f16/bf16
  float* lse;        // [B, Hq, N] fp32 or nullptr
  int B, Hq, Hkv, N;
  int group;         // Hq / Hkv
  int n_qpairs;      // ceil(N / 256): CTAs per (batch, head)
  int n_kv_tiles;    // ceil(N / 128)
  int causal;
  float scale_log2;  // scale * log2(e)
  int debug_flags;
  long long* trace;  // timeline samples, used only in FA_TRACE builds
  unsigned epoch;    // launch counter, tags device status words
  unsigned long long timeout_ns;
};

cudaError_t launch_fwd(const FwdParams& p, int head_dim, bool bf16, cudaStream_t stream);
int smem_bytes_for(int head_dim);
cudaError_t read_status(unsigned long long* out, bool reset);

}  // namespace fa
