// pybind module `flash_attn_sm75_cuda` — the reference's L3 binding
// (src/bindings/pytorch_extension.cpp:1-129) re-implemented over the C ABI in
// include/fa_b200.h.  Same four exported functions with the same argument
// lists and input checks; the kernels run asynchronously on PyTorch's
// current CUDA stream instead of the legacy stream + cudaDeviceSynchronize.
//
// Additions: native GQA (K/V may have fewer heads than Q), bf16 inputs,
// flash_attention_forward_lse returning (O, LSE), flash_attention_forward_kvcache
// (Nq != Nk: decode and chunked prefill), and diagnostics.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "fa_b200.h"

namespace {

void check_tensor(const torch::Tensor& t, const char* name, bool allow_bf16) {
  TORCH_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  if (allow_bf16) {
    TORCH_CHECK(t.dtype() == torch::kFloat16 || t.dtype() == torch::kBFloat16,
                std::string(name) + " must be FP16 or BF16");
  } else {
    TORCH_CHECK(t.dtype() == torch::kFloat16, std::string(name) + " must be FP16");
  }
  TORCH_CHECK(t.is_contiguous(), std::string(name) + " must be contiguous");
  TORCH_CHECK(t.dim() == 4, std::string(name) + " must be [B, H, N, D]");
}

void* stream_of(const torch::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

std::tuple<torch::Tensor, torch::Tensor> fwd_impl(const torch::Tensor& Q, const torch::Tensor& K,
                                                  const torch::Tensor& V, bool causal, float scale,
                                                  bool want_lse) {
  check_tensor(Q, "Q", true);
  check_tensor(K, "K", true);
  check_tensor(V, "V", true);
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype(), "Q, K, V must share a dtype");
  TORCH_CHECK(Q.device() == K.device() && Q.device() == V.device(),
              "Q, K, V must be on the same device");
  TORCH_CHECK(Q.size(0) == K.size(0), "batch mismatch");
  TORCH_CHECK(Q.size(2) == K.size(2), "seq_len mismatch");
  TORCH_CHECK(Q.size(3) == K.size(3), "head_dim mismatch");
  TORCH_CHECK(K.sizes() == V.sizes(), "K and V must have identical shapes");
  const auto head_dim = Q.size(3);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  TORCH_CHECK(Q.size(0) <= INT32_MAX && Q.size(1) <= INT32_MAX && Q.size(2) <= INT32_MAX,
              "size exceeds int32");

  const c10::cuda::CUDAGuard guard(Q.device());
  auto O = torch::empty_like(Q);
  torch::Tensor lse;
  if (want_lse)
    lse = torch::empty({Q.size(0), Q.size(1), Q.size(2)},
                       Q.options().dtype(torch::kFloat32));
  const int rc = fa_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                        want_lse ? lse.data_ptr<float>() : nullptr, static_cast<int>(Q.size(0)),
                        static_cast<int>(Q.size(1)), static_cast<int>(K.size(1)),
                        static_cast<int>(Q.size(2)), static_cast<int>(head_dim), scale,
                        causal ? 1 : 0,
                        Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16,
                        stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_forward: ", fa_error_string(rc));
  return {O, lse};
}

// Forward into caller-provided O (and optional LSE) on the current stream;
// used by the host-buffer pipeline, which computes per-chunk slices in place.
void flash_attention_forward_out(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                 torch::Tensor O, c10::optional<torch::Tensor> lse, bool causal,
                                 float scale) {
  check_tensor(Q, "Q", true);
  check_tensor(K, "K", true);
  check_tensor(V, "V", true);
  check_tensor(O, "O", true);
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype() && Q.dtype() == O.dtype(),
              "Q, K, V, O must share a dtype");
  TORCH_CHECK(Q.device() == K.device() && Q.device() == V.device() && Q.device() == O.device(),
              "Q, K, V, O must be on the same device");
  TORCH_CHECK(O.sizes() == Q.sizes(), "O must have Q's shape");
  TORCH_CHECK(Q.size(0) == K.size(0) && Q.size(2) == K.size(2) && Q.size(3) == K.size(3),
              "Q and K shapes differ beyond the head count");
  TORCH_CHECK(K.sizes() == V.sizes(), "K and V must have identical shapes");
  const auto head_dim = Q.size(3);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  float* lse_ptr = nullptr;
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->is_cuda() && lse->dtype() == torch::kFloat32 && lse->is_contiguous() &&
                    lse->dim() == 3 && lse->size(0) == Q.size(0) && lse->size(1) == Q.size(1) &&
                    lse->size(2) == Q.size(2),
                "lse must be a contiguous fp32 CUDA tensor [B, Hq, N]");
    lse_ptr = lse->data_ptr<float>();
  }
  TORCH_CHECK(Q.size(0) <= INT32_MAX && Q.size(1) <= INT32_MAX && Q.size(2) <= INT32_MAX,
              "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  const int rc = fa_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse_ptr,
                        static_cast<int>(Q.size(0)), static_cast<int>(Q.size(1)),
                        static_cast<int>(K.size(1)), static_cast<int>(Q.size(2)),
                        static_cast<int>(head_dim), scale, causal ? 1 : 0,
                        Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16,
                        stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_forward: ", fa_error_string(rc));
}

torch::Tensor flash_attention_forward(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                      bool causal, float scale) {
  return std::get<0>(fwd_impl(Q, K, V, causal, scale, false));
}

std::tuple<torch::Tensor, torch::Tensor> flash_attention_forward_lse(torch::Tensor Q,
                                                                     torch::Tensor K,
                                                                     torch::Tensor V, bool causal,
                                                                     float scale) {
  return fwd_impl(Q, K, V, causal, scale, true);
}

// Reference ablation exports (d=64, identical shapes): one kernel serves all.
torch::Tensor d64_variant(const char* what, torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                          bool causal, float scale) {
  check_tensor(Q, "Q", false);
  check_tensor(K, "K", false);
  check_tensor(V, "V", false);
  TORCH_CHECK(Q.sizes() == K.sizes() && Q.sizes() == V.sizes(),
              "Q, K, V must have identical shapes");
  TORCH_CHECK(Q.size(3) == 64, std::string(what) + " kernel supports head_dim=64 only");
  return flash_attention_forward(Q, K, V, causal, scale);
}

torch::Tensor flash_attention_forward_scalar(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                             bool causal, float scale) {
  return d64_variant("scalar", Q, K, V, causal, scale);
}

torch::Tensor flash_attention_forward_wmma_qk(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                              bool causal, float scale) {
  return d64_variant("wmma_qk", Q, K, V, causal, scale);
}

torch::Tensor naive_attention_forward(torch::Tensor Q, torch::Tensor K, torch::Tensor V,
                                      bool causal, float scale) {
  check_tensor(Q, "Q", false);
  check_tensor(K, "K", false);
  check_tensor(V, "V", false);
  TORCH_CHECK(Q.sizes() == K.sizes() && Q.sizes() == V.sizes(),
              "naive_attention: Q, K, V must have identical shapes");
  const c10::cuda::CUDAGuard guard(Q.device());
  auto O = torch::empty_like(Q);
  auto ws = torch::empty({Q.size(0) * Q.size(1), Q.size(2), Q.size(2)},
                         Q.options().dtype(torch::kFloat32));
  const int rc = fa_naive_fwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                              static_cast<int>(Q.size(0)), static_cast<int>(Q.size(1)),
                              static_cast<int>(Q.size(2)), static_cast<int>(Q.size(3)), scale,
                              causal ? 1 : 0, ws.data_ptr<float>(), stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "naive_attention_forward: ", fa_error_string(rc));
  return O;
}

// Nq new queries against Nk cached keys (decode / chunked prefill); causal is
// an FA_CAUSAL_* mode.  The split-KV workspace comes from PyTorch's caching
// allocator on the current stream.  Returns (O, LSE).
std::tuple<torch::Tensor, torch::Tensor> flash_attention_forward_kvcache(
    torch::Tensor Q, torch::Tensor K, torch::Tensor V, int64_t causal, float scale) {
  check_tensor(Q, "Q", true);
  check_tensor(K, "K", true);
  check_tensor(V, "V", true);
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype(), "Q, K, V must share a dtype");
  TORCH_CHECK(Q.device() == K.device() && Q.device() == V.device(),
              "Q, K, V must be on the same device");
  TORCH_CHECK(Q.size(0) == K.size(0), "batch mismatch");
  TORCH_CHECK(Q.size(3) == K.size(3), "head_dim mismatch");
  TORCH_CHECK(K.sizes() == V.sizes(), "K and V must have identical shapes");
  const auto head_dim = Q.size(3);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  TORCH_CHECK(causal >= FA_CAUSAL_NONE && causal <= FA_CAUSAL_TOP_LEFT, "bad causal mode ", causal);
  TORCH_CHECK(Q.size(0) <= INT32_MAX && Q.size(1) <= INT32_MAX && Q.size(2) <= INT32_MAX &&
                  K.size(2) <= INT32_MAX,
              "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  const int B = static_cast<int>(Q.size(0)), Hq = static_cast<int>(Q.size(1));
  const int Hkv = static_cast<int>(K.size(1)), Nq = static_cast<int>(Q.size(2));
  const int Nk = static_cast<int>(K.size(2)), d = static_cast<int>(head_dim);
  auto O = torch::empty_like(Q);
  auto lse = torch::empty({Q.size(0), Q.size(1), Q.size(2)}, Q.options().dtype(torch::kFloat32));
  const size_t ws_bytes = fa_fwd_kvcache_workspace_bytes(B, Hq, Hkv, Nq, Nk, d);
  torch::Tensor ws;
  if (ws_bytes > 0)
    ws = torch::empty({static_cast<int64_t>(ws_bytes)}, Q.options().dtype(torch::kUInt8));
  const int rc = fa_fwd_kvcache(
      Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse.data_ptr<float>(), B, Hq, Hkv,
      Nq, Nk, d, scale, static_cast<int>(causal),
      Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16,
      ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes, stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_forward_kvcache: ", fa_error_string(rc));
  return {O, lse};
}

void check_rows(const torch::Tensor& t, const char* name, int64_t n, const torch::Tensor& like) {
  TORCH_CHECK(t.is_cuda() && t.device() == like.device(), std::string(name) +
                                                              " must be on the inputs' device");
  TORCH_CHECK(t.dtype() == torch::kInt32 && t.dim() == 1 && t.is_contiguous() && t.size(0) == n,
              std::string(name) + " must be a contiguous int32 tensor of ", n, " entries");
}

void check_packed(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  TORCH_CHECK(t.dtype() == torch::kFloat16 || t.dtype() == torch::kBFloat16,
              std::string(name) + " must be FP16 or BF16");
  TORCH_CHECK(t.is_contiguous(), std::string(name) + " must be contiguous");
  TORCH_CHECK(t.dim() == 3, std::string(name) + " must be [total, H, D]");
}

// Packed variable-length batch: Q [total_q, Hq, d], K/V [total_k, Hkv, d],
// cu_seqlens_* int32 [B + 1] on the device.  Returns O [total_q, Hq, d] and
// LSE fp32 [Hq, total_q].
std::tuple<torch::Tensor, torch::Tensor> flash_attention_forward_varlen(
    torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor cu_seqlens_q,
    torch::Tensor cu_seqlens_k, int64_t max_seqlen_q, int64_t max_seqlen_k, int64_t causal,
    float scale) {
  check_packed(Q, "Q");
  check_packed(K, "K");
  check_packed(V, "V");
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype(), "Q, K, V must share a dtype");
  TORCH_CHECK(Q.device() == K.device() && Q.device() == V.device(),
              "Q, K, V must be on the same device");
  TORCH_CHECK(K.sizes() == V.sizes(), "K and V must have identical shapes");
  TORCH_CHECK(Q.size(2) == K.size(2), "head_dim mismatch");
  const auto head_dim = Q.size(2);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  TORCH_CHECK(causal >= FA_CAUSAL_NONE && causal <= FA_CAUSAL_TOP_LEFT, "bad causal mode ", causal);
  TORCH_CHECK(cu_seqlens_q.dim() == 1 && cu_seqlens_q.size(0) >= 1,
              "cu_seqlens_q must be [B + 1]");
  const int64_t B = cu_seqlens_q.size(0) - 1;
  check_rows(cu_seqlens_q, "cu_seqlens_q", B + 1, Q);
  check_rows(cu_seqlens_k, "cu_seqlens_k", B + 1, Q);
  TORCH_CHECK(Q.size(0) <= INT32_MAX && K.size(0) <= INT32_MAX && max_seqlen_q >= 0 &&
                  max_seqlen_q <= INT32_MAX && max_seqlen_k >= 0 && max_seqlen_k <= INT32_MAX,
              "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  auto O = torch::zeros_like(Q);
  auto lse = torch::full({Q.size(1), Q.size(0)}, -INFINITY, Q.options().dtype(torch::kFloat32));
  const int rc = fa_fwd_varlen(
      Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse.data_ptr<float>(),
      cu_seqlens_q.data_ptr<int>(), cu_seqlens_k.data_ptr<int>(), static_cast<int>(B),
      static_cast<int>(Q.size(1)), static_cast<int>(K.size(1)), static_cast<int>(Q.size(0)),
      static_cast<int>(K.size(0)), static_cast<int>(max_seqlen_q), static_cast<int>(max_seqlen_k),
      static_cast<int>(head_dim), scale, static_cast<int>(causal),
      Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16, stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_forward_varlen: ", fa_error_string(rc));
  return {O, lse};
}

// Padded batch: Q [B, Hq, Nq, d], K/V [B, Hkv, Nk, d] and per batch entry the
// valid query rows [q_start, q_end) and key rows [k_start, k_end) (int32 [B]
// on the device).  Rows outside a query range come back as O = 0, LSE = -inf.
std::tuple<torch::Tensor, torch::Tensor> flash_attention_forward_padded(
    torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor q_start, torch::Tensor q_end,
    torch::Tensor k_start, torch::Tensor k_end, int64_t causal, float scale) {
  check_tensor(Q, "Q", true);
  check_tensor(K, "K", true);
  check_tensor(V, "V", true);
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype(), "Q, K, V must share a dtype");
  TORCH_CHECK(Q.device() == K.device() && Q.device() == V.device(),
              "Q, K, V must be on the same device");
  TORCH_CHECK(Q.size(0) == K.size(0), "batch mismatch");
  TORCH_CHECK(Q.size(3) == K.size(3), "head_dim mismatch");
  TORCH_CHECK(K.sizes() == V.sizes(), "K and V must have identical shapes");
  const auto head_dim = Q.size(3);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  TORCH_CHECK(causal >= FA_CAUSAL_NONE && causal <= FA_CAUSAL_TOP_LEFT, "bad causal mode ", causal);
  const int64_t B = Q.size(0);
  check_rows(q_start, "q_start", B, Q);
  check_rows(q_end, "q_end", B, Q);
  check_rows(k_start, "k_start", B, Q);
  check_rows(k_end, "k_end", B, Q);
  TORCH_CHECK(Q.size(0) <= INT32_MAX && Q.size(1) <= INT32_MAX && Q.size(2) <= INT32_MAX &&
                  K.size(2) <= INT32_MAX,
              "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  auto O = torch::zeros_like(Q);
  auto lse = torch::full({Q.size(0), Q.size(1), Q.size(2)}, -INFINITY,
                         Q.options().dtype(torch::kFloat32));
  const int rc = fa_fwd_padded(
      Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), lse.data_ptr<float>(),
      q_start.data_ptr<int>(), q_end.data_ptr<int>(), k_start.data_ptr<int>(),
      k_end.data_ptr<int>(), static_cast<int>(B), static_cast<int>(Q.size(1)),
      static_cast<int>(K.size(1)), static_cast<int>(Q.size(2)), static_cast<int>(K.size(2)),
      static_cast<int>(head_dim), scale, static_cast<int>(causal),
      Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16, stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_forward_padded: ", fa_error_string(rc));
  return {O, lse};
}

// Gradients of flash_attention_forward_lse: (dQ, dK, dV) from dO, the inputs,
// the forward's O and LSE.  The workspace comes from PyTorch's allocator.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> flash_attention_backward(
    torch::Tensor dO, torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor O,
    torch::Tensor lse, bool causal, float scale) {
  check_tensor(Q, "Q", true);
  check_tensor(K, "K", true);
  check_tensor(V, "V", true);
  check_tensor(O, "O", true);
  check_tensor(dO, "dO", true);
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype() && Q.dtype() == O.dtype() &&
                  Q.dtype() == dO.dtype(),
              "Q, K, V, O, dO must share a dtype");
  TORCH_CHECK(O.sizes() == Q.sizes() && dO.sizes() == Q.sizes(), "O and dO must have Q's shape");
  TORCH_CHECK(K.sizes() == V.sizes() && Q.size(0) == K.size(0) && Q.size(2) == K.size(2) &&
                  Q.size(3) == K.size(3),
              "K, V shapes do not match Q");
  TORCH_CHECK(lse.is_cuda() && lse.dtype() == torch::kFloat32 && lse.is_contiguous() &&
                  lse.dim() == 3 && lse.size(0) == Q.size(0) && lse.size(1) == Q.size(1) &&
                  lse.size(2) == Q.size(2),
              "lse must be a contiguous fp32 CUDA tensor [B, Hq, N]");
  const auto head_dim = Q.size(3);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  TORCH_CHECK(Q.size(0) <= INT32_MAX && Q.size(1) <= INT32_MAX && Q.size(2) <= INT32_MAX,
              "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  const int B = static_cast<int>(Q.size(0)), Hq = static_cast<int>(Q.size(1));
  const int N = static_cast<int>(Q.size(2));
  auto dQ = torch::empty_like(Q);
  auto dK = torch::empty_like(K);
  auto dV = torch::empty_like(V);
  const size_t ws_bytes = fa_bwd_workspace_bytes(B, Hq, N);
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 16)},
                         Q.options().dtype(torch::kUInt8));
  const int rc = fa_bwd(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), dO.data_ptr(),
                        lse.data_ptr<float>(), dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), B, Hq,
                        static_cast<int>(K.size(1)), N, static_cast<int>(head_dim), scale,
                        causal ? 1 : 0, Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16,
                        ws.data_ptr(), ws_bytes, stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_backward: ", fa_error_string(rc));
  return {dQ, dK, dV};
}

// Gradients of flash_attention_forward_padded (square N): (dQ, dK, dV).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> flash_attention_backward_padded(
    torch::Tensor dO, torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor O,
    torch::Tensor lse, torch::Tensor q_start, torch::Tensor q_end, torch::Tensor k_start,
    torch::Tensor k_end, bool causal, float scale) {
  check_tensor(Q, "Q", true);
  check_tensor(K, "K", true);
  check_tensor(V, "V", true);
  check_tensor(O, "O", true);
  check_tensor(dO, "dO", true);
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype() && Q.dtype() == O.dtype() &&
                  Q.dtype() == dO.dtype(),
              "Q, K, V, O, dO must share a dtype");
  TORCH_CHECK(O.sizes() == Q.sizes() && dO.sizes() == Q.sizes(), "O and dO must have Q's shape");
  TORCH_CHECK(K.sizes() == V.sizes() && Q.size(0) == K.size(0) && Q.size(2) == K.size(2) &&
                  Q.size(3) == K.size(3),
              "K, V shapes do not match Q (the padded backward needs Nq = Nk)");
  TORCH_CHECK(lse.is_cuda() && lse.dtype() == torch::kFloat32 && lse.is_contiguous() &&
                  lse.dim() == 3 && lse.size(0) == Q.size(0) && lse.size(1) == Q.size(1) &&
                  lse.size(2) == Q.size(2),
              "lse must be a contiguous fp32 CUDA tensor [B, Hq, N]");
  const auto head_dim = Q.size(3);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  const int64_t B = Q.size(0);
  check_rows(q_start, "q_start", B, Q);
  check_rows(q_end, "q_end", B, Q);
  check_rows(k_start, "k_start", B, Q);
  check_rows(k_end, "k_end", B, Q);
  TORCH_CHECK(Q.size(1) <= INT32_MAX && Q.size(2) <= INT32_MAX, "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  const int Hq = static_cast<int>(Q.size(1)), N = static_cast<int>(Q.size(2));
  auto dQ = torch::empty_like(Q);
  auto dK = torch::empty_like(K);
  auto dV = torch::empty_like(V);
  const size_t ws_bytes = fa_bwd_workspace_bytes(static_cast<int>(B), Hq, N);
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 16)},
                         Q.options().dtype(torch::kUInt8));
  const int rc = fa_bwd_padded(
      Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), dO.data_ptr(), lse.data_ptr<float>(),
      q_start.data_ptr<int>(), q_end.data_ptr<int>(), k_start.data_ptr<int>(), k_end.data_ptr<int>(),
      dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), static_cast<int>(B), Hq,
      static_cast<int>(K.size(1)), N, static_cast<int>(head_dim), scale, causal ? 1 : 0,
      Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16, ws.data_ptr(), ws_bytes,
      stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_backward_padded: ", fa_error_string(rc));
  return {dQ, dK, dV};
}

// Gradients of flash_attention_forward_varlen for packed self-attention batches.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> flash_attention_backward_varlen(
    torch::Tensor dO, torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor O,
    torch::Tensor lse, torch::Tensor cu_seqlens, int64_t max_seqlen, bool causal, float scale) {
  check_packed(Q, "Q");
  check_packed(K, "K");
  check_packed(V, "V");
  check_packed(O, "O");
  check_packed(dO, "dO");
  TORCH_CHECK(Q.dtype() == K.dtype() && Q.dtype() == V.dtype() && Q.dtype() == O.dtype() &&
                  Q.dtype() == dO.dtype(),
              "Q, K, V, O, dO must share a dtype");
  TORCH_CHECK(O.sizes() == Q.sizes() && dO.sizes() == Q.sizes(), "O and dO must have Q's shape");
  TORCH_CHECK(K.sizes() == V.sizes() && K.size(0) == Q.size(0) && K.size(2) == Q.size(2),
              "K, V must be [total, Hkv, d] over the same rows as Q (self-attention)");
  TORCH_CHECK(lse.is_cuda() && lse.dtype() == torch::kFloat32 && lse.is_contiguous() &&
                  lse.dim() == 2 && lse.size(0) == Q.size(1) && lse.size(1) == Q.size(0),
              "lse must be a contiguous fp32 CUDA tensor [Hq, total]");
  const auto head_dim = Q.size(2);
  TORCH_CHECK(head_dim == 64 || head_dim == 128,
              "flash_attention_forward supports head_dim=64 or 128, got ", head_dim);
  TORCH_CHECK(K.size(1) > 0 && Q.size(1) % K.size(1) == 0, "GQA: Q heads (", Q.size(1),
              ") not divisible by K/V heads (", K.size(1), ")");
  TORCH_CHECK(cu_seqlens.dim() == 1 && cu_seqlens.size(0) >= 1, "cu_seqlens must be [B + 1]");
  const int64_t B = cu_seqlens.size(0) - 1;
  check_rows(cu_seqlens, "cu_seqlens", B + 1, Q);
  TORCH_CHECK(Q.size(0) <= INT32_MAX && max_seqlen >= 0 && max_seqlen <= INT32_MAX,
              "size exceeds int32");
  const c10::cuda::CUDAGuard guard(Q.device());
  const int Hq = static_cast<int>(Q.size(1));
  auto dQ = torch::empty_like(Q);
  auto dK = torch::empty_like(K);
  auto dV = torch::empty_like(V);
  const size_t ws_bytes = fa_bwd_workspace_bytes(static_cast<int>(B), Hq, static_cast<int>(max_seqlen));
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 16)},
                         Q.options().dtype(torch::kUInt8));
  const int rc = fa_bwd_varlen(
      Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), dO.data_ptr(), lse.data_ptr<float>(),
      cu_seqlens.data_ptr<int>(), dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), static_cast<int>(B),
      Hq, static_cast<int>(K.size(1)), static_cast<int>(Q.size(0)), static_cast<int>(max_seqlen),
      static_cast<int>(head_dim), scale, causal ? 1 : 0,
      Q.dtype() == torch::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16, ws.data_ptr(), ws_bytes,
      stream_of(Q));
  TORCH_CHECK(rc == FA_OK, "flash_attention_backward_varlen: ", fa_error_string(rc));
  return {dQ, dK, dV};
}

int device_status(bool reset) { return fa_device_status(reset ? 1 : 0); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("naive_attention_forward", &naive_attention_forward);
  m.def("flash_attention_forward", &flash_attention_forward);
  m.def("flash_attention_forward_scalar", &flash_attention_forward_scalar);
  m.def("flash_attention_forward_wmma_qk", &flash_attention_forward_wmma_qk);
  m.def("flash_attention_forward_lse", &flash_attention_forward_lse,
        "Returns (O, LSE) with LSE fp32 [B, Hq, N]");
  m.def("flash_attention_forward_out", &flash_attention_forward_out, pybind11::arg("Q"),
        pybind11::arg("K"), pybind11::arg("V"), pybind11::arg("O"), pybind11::arg("lse"),
        pybind11::arg("causal"), pybind11::arg("scale"));
  m.def("flash_attention_backward", &flash_attention_backward,
        "(dQ, dK, dV) from dO, Q, K, V, O, LSE (fp32 [B, Hq, N]), causal, scale");
  m.def("flash_attention_forward_kvcache", &flash_attention_forward_kvcache,
        "O, LSE of Nq queries against Nk cached keys; causal: 0 none, 1 bottom-right, 2 top-left");
  m.def("flash_attention_forward_varlen", &flash_attention_forward_varlen,
        "(O [total_q, Hq, d], LSE [Hq, total_q]) of a packed variable-length batch");
  m.def("flash_attention_forward_padded", &flash_attention_forward_padded,
        "(O, LSE) of a padded batch with per-entry valid query / key row ranges");
  m.def("flash_attention_backward_padded", &flash_attention_backward_padded,
        "(dQ, dK, dV) of flash_attention_forward_padded for square padded batches");
  m.def("flash_attention_backward_varlen", &flash_attention_backward_varlen,
        "(dQ, dK, dV) of flash_attention_forward_varlen for packed self-attention batches");
  m.def("device_status", &device_status, pybind11::arg("reset") = false,
        "Error code recorded by the in-kernel watchdog (0 = none)");
  m.def("set_watchdog_ns", &fa_set_watchdog_ns);
  m.def("set_debug_flags", &fa_set_debug_flags);
  m.def("smem_bytes", &fa_smem_bytes);
  m.def("version", []() { return std::string(fa_version()); });
}
