/*
 * fa_b200.h — C ABI of the B200 (sm_100a) FlashAttention forward.
 *
 * Drop-in boundary for the reference's attention-forward path
 * (JohnScheuer/flash-attention-sm75-register-fused).  Every entry point takes
 * plain device pointers and sizes; no framework types cross this boundary.
 *
 * Layout (all entry points): Q [B, Hq, N, d], K/V [B, Hkv, N, d], O like Q,
 * row-major and contiguous, f16 (or bf16 where a dtype argument exists).
 * LSE (optional) is fp32 [B, Hq, N], natural log:  LSE = log sum_j exp(s_ij).
 * Causal masking is top-left aligned: query i attends keys j <= i.
 * GQA: query head h reads KV head h / (Hq / Hkv) (repeat_interleave order).
 *
 * Pointer arguments are typed void* here; the reference declares the legacy
 * launchers with `half*`, which is the same C ABI, so the reference binding
 * (src/bindings/pytorch_extension.cpp:4-19) links against this library as is.
 */
#ifndef FA_B200_H
#define FA_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes returned by the int-returning entry points ---- */
enum {
  FA_OK = 0,
  FA_ERR_INVALID_ARG = 1,          /* null pointer, negative size, bad causal/dtype flag */
  FA_ERR_UNSUPPORTED_HEAD_DIM = 2, /* head_dim not in {64, 128} */
  FA_ERR_GQA_DIVISIBILITY = 3,     /* Hq % Hkv != 0 */
  FA_ERR_ALIGNMENT = 4,            /* a pointer is not 16-byte aligned */
  FA_ERR_DTYPE = 5,                /* dtype not FA_DTYPE_F16 / FA_DTYPE_BF16 */
  FA_ERR_TENSOR_MAP = 6,           /* cuTensorMapEncodeTiled rejected a shape */
  FA_ERR_LAUNCH = 7,               /* kernel launch failed (see cudaGetLastError) */
  FA_ERR_DEVICE = 8,               /* current device is not sm_100 */
  FA_ERR_CUDA = 9,                 /* another CUDA runtime call failed */
  FA_ERR_TOO_LARGE = 10,           /* a size overflows the kernel's index types */
  FA_ERR_SCRATCH_LIMIT = 11,       /* fa_naive_fwd_noalloc: problem larger than its static scratch */
  FA_ERR_TIMEOUT_BASE = 100        /* device watchdog: 100 + wait site id */
};

enum { FA_DTYPE_F16 = 0, FA_DTYPE_BF16 = 1 };

/* Causal alignment for fa_fwd_kvcache (fa_fwd takes 0/1; for Nq == Nk both
 * alignments are the reference's top-left mask, attention_ref.py:33-40). */
enum {
  FA_CAUSAL_NONE = 0,
  FA_CAUSAL_BOTTOM_RIGHT = 1, /* key j visible to query i iff j <= i + Nk - Nq (KV cache) */
  FA_CAUSAL_TOP_LEFT = 2      /* key j visible to query i iff j <= i (SDPA is_causal) */
};

/* Test hooks (fa_set_debug_flags). */
enum {
  FA_DEBUG_SKIP_Q_LOAD = 1, /* producer never loads Q: the consumers' wait must time out */
  FA_DEBUG_PAIR_KERNEL = 2, /* square / chunked prefill always on the pair kernel (two Q
                               tiles per CTA), for comparisons */
  FA_DEBUG_TILE_SPLIT2 = 4, /* tile kernel with each tile's keys split between 2 softmax
                               warpgroups instead of 4, for comparisons */
  FA_DEBUG_TILE_KERNEL = 8, /* square / chunked prefill always on the tile kernel (one Q
                               tile per CTA, S double-buffered), for comparisons */
  FA_DEBUG_PAIR2_KERNEL = 16, /* d = 128 square / chunked prefill on CTA pairs (one product
                                for two SMs) wherever they apply (opt-in) */
  FA_DEBUG_NO_TAIL_SPLIT = 32, /* keep a pair-kernel launch's half-empty last wave on the pair
                                 kernel instead of the tile kernel, for comparisons */
  FA_DEBUG_NO_PERSIST = 64,     /* one CTA per pair-kernel work item instead of persistent
                                 CTAs, for comparisons */
  FA_DEBUG_STATIC_DEAL = 128,   /* persistent pair-kernel CTAs deal every round in the fixed
                                 boustrophedon order (the last rounds too), for comparisons */
  FA_DEBUG_DUAL_TILES = 256     /* d = 64 square launches as one-Q-tile items whose two softmax
                                 groups split the keys and merge in the CTA, wherever they apply
                                 (by default only non-causal launches of one to two waves of Q
                                 pairs; FA_DEBUG_PAIR_KERNEL keeps Q pairs there) */
};

/*
 * fa_fwd — asynchronous attention forward on `stream` (cudaStream_t; NULL =
 * legacy default stream).  Returns FA_OK or an FA_ERR_* code; argument errors
 * are reported before anything is launched.  B == 0, Hq == 0 or N == 0 is a
 * no-op.  `lse` may be NULL.
 *
 * Replaces: launch_flash_attention_forward
 *   (reference src/kernels/flash_attention_forward.cu:795-817) with native
 *   GQA (reference expands K/V in src/flash_attention_sm75/ops.py:6-27),
 *   an LSE output, bf16, a caller stream and an error code.
 */
int fa_fwd(const void* Q, const void* K, const void* V, void* O, float* lse, int B, int Hq,
           int Hkv, int N, int head_dim, float scale, int causal, int dtype, void* stream);

/*
 * fa_fwd_kvcache — attention of Nq new queries against Nk cached keys
 * (decode: Nq = 1; chunked prefill: Nq < Nk).  Q/O are [B, Hq, Nq, d], K/V
 * [B, Hkv, Nk, d], LSE [B, Hq, Nq]; `causal` is an FA_CAUSAL_* value.  Rows
 * that see no key (bottom-right with Nq > Nk) get O = 0 and LSE = -inf.
 * When the call alone would not fill the GPU, the key range is split across
 * CTAs and merged by a second kernel; that needs `workspace` (16-byte aligned)
 * of at least fa_fwd_kvcache_workspace_bytes() bytes, otherwise (NULL or
 * smaller) the call runs unsplit.  Asynchronous on `stream`.
 *
 * No reference counterpart: the reference's HF patch sends these calls to
 * PyTorch SDPA (reference src/flash_attention_sm75/llama_attention_replacement.py:63-65,
 * reason "kvcache_decode").
 */
int fa_fwd_kvcache(const void* Q, const void* K, const void* V, void* O, float* lse, int B,
                   int Hq, int Hkv, int Nq, int Nk, int head_dim, float scale, int causal,
                   int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes fa_fwd_kvcache needs to split this problem (0: no split). */
size_t fa_fwd_kvcache_workspace_bytes(int B, int Hq, int Hkv, int Nq, int Nk, int head_dim);

/*
 * fa_fwd_varlen — attention over a packed batch of variable-length sequences
 * (the cu_seqlens layout): Q/O [total_q, Hq, d], K/V [total_k, Hkv, d], all
 * contiguous.  Sequence b owns query rows [cu_seqlens_q[b], cu_seqlens_q[b+1])
 * and key rows [cu_seqlens_k[b], cu_seqlens_k[b+1]); the offsets are int32
 * DEVICE arrays of B + 1 non-decreasing entries (clamped to [0, total]).
 * max_seqlen_q / max_seqlen_k bound the lengths (query rows of a longer
 * sequence past max_seqlen_q, rounded up to 256, are not computed).
 * `causal`: FA_CAUSAL_BOTTOM_RIGHT (key j visible to query i of a sequence iff
 * j <= i + nk - nq), FA_CAUSAL_TOP_LEFT (j <= i) or FA_CAUSAL_NONE.  LSE (may be
 * NULL) is fp32 [Hq, total_q].  Rows that see no key get O = 0, LSE = -inf.
 * Keys past a sequence's end are masked; the V rows that follow it in the
 * packed buffer (the next sequence's) are multiplied by exactly 0, so they
 * must be finite.  Asynchronous on `stream`.
 *
 * No reference counterpart: the reference's HF patch sends masked (padded /
 * varlen) batches to PyTorch SDPA (reference
 * src/flash_attention_sm75/llama_attention_replacement.py:61-62, reason
 * "has_attn_mask").
 */
int fa_fwd_varlen(const void* Q, const void* K, const void* V, void* O, float* lse,
                  const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                  int total_q, int total_k, int max_seqlen_q, int max_seqlen_k, int head_dim,
                  float scale, int causal, int dtype, void* stream);

/*
 * fa_fwd_padded — attention of a padded batch in the fixed layout (Q/O
 * [B, Hq, Nq, d], K/V [B, Hkv, Nk, d], LSE [B, Hq, Nq]): batch entry b's valid
 * queries are rows [q_start[b], q_end[b]) and its valid keys rows
 * [k_start[b], k_end[b]) (int32 DEVICE arrays of B entries, clamped to
 * [0, Nq] / [0, Nk]).  Padding keys are never attended; rows of O and LSE
 * outside a query range are not written.  `causal` follows fa_fwd_kvcache on
 * the full padded rows (BOTTOM_RIGHT: key j visible to query i iff
 * j <= i + Nk - Nq; TOP_LEFT: j <= i), restricted to the valid keys; valid
 * rows that then see no key get O = 0, LSE = -inf.  Covers left padding
 * (start > 0), right padding (end < N) and both.  Asynchronous on `stream`.
 *
 * No reference counterpart (reference llama_attention_replacement.py:61-62).
 */
int fa_fwd_padded(const void* Q, const void* K, const void* V, void* O, float* lse,
                  const int* q_start, const int* q_end, const int* k_start, const int* k_end,
                  int B, int Hq, int Hkv, int Nq, int Nk, int head_dim, float scale, int causal,
                  int dtype, void* stream);

/*
 * fa_bwd — gradients of fa_fwd (square, causal 0/1 top-left, GQA): from Q, K, V,
 * the forward's O and LSE ([B, Hq, N] fp32, natural log) and dO = dL/dO, writes
 * dQ [B, Hq, N, d], dK and dV [B, Hkv, N, d] (GQA: summed over each group's
 * query heads).  `workspace` (16-byte aligned) needs fa_bwd_workspace_bytes()
 * bytes.  Asynchronous on `stream`; same error codes as fa_fwd.
 *
 * No reference counterpart: the reference's autograd Function raises in
 * backward (reference src/flash_attention_sm75/ops.py:47-52).
 */
int fa_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
           const float* lse, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv, int N,
           int head_dim, float scale, int causal, int dtype, void* workspace,
           size_t workspace_bytes, void* stream);

/* Workspace bytes of fa_bwd: two fp32 values per query row (from LSE and rowsum(dO*O)) and two
 * 4 KB operand tiles per 128-row query tile, rows padded to 128. */
size_t fa_bwd_workspace_bytes(int B, int Hq, int N);

/*
 * fa_bwd_padded — gradients of fa_fwd_padded for square padded batches
 * (Nq = Nk = N): batch entry b's valid query rows are [q_start[b], q_end[b]) and
 * valid keys [k_start[b], k_end[b]) (int32 device arrays of B entries); O and
 * LSE come from fa_fwd_padded (rows outside a query range: O = 0, LSE = -inf, as
 * the Python API returns them).  Padding keys get dK = dV = 0 and query rows
 * outside the ranges dQ = 0.  `causal` 0/1 (bottom-right = top-left for square
 * inputs).  Workspace, errors and stream as fa_bwd.
 *
 * No reference counterpart (reference llama_attention_replacement.py:61-62).
 */
int fa_bwd_padded(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                  const float* lse, const int* q_start, const int* q_end, const int* k_start,
                  const int* k_end, void* dQ, void* dK, void* dV, int B, int Hq, int Hkv, int N,
                  int head_dim, float scale, int causal, int dtype, void* workspace,
                  size_t workspace_bytes, void* stream);

/*
 * fa_bwd_varlen — gradients of fa_fwd_varlen for packed self-attention batches
 * (the same cu_seqlens for queries and keys): Q, K, V, O, dO, dQ, dK, dV in the
 * packed layout ([total, H, d]), LSE fp32 [Hq, total] from fa_fwd_varlen,
 * cu_seqlens int32 device array of B + 1 offsets, max_seqlen >= every length.
 * `causal` 0/1.  Workspace: fa_bwd_workspace_bytes(B, Hq, max_seqlen).
 * Errors and stream as fa_bwd.
 *
 * No reference counterpart (reference llama_attention_replacement.py:61-62).
 */
int fa_bwd_varlen(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                  const float* lse, const int* cu_seqlens, void* dQ, void* dK, void* dV, int B,
                  int Hq, int Hkv, int total, int max_seqlen, int head_dim, float scale,
                  int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ---- reference-compatible launchers (void, fp16, blocking) ----
 * Same signatures and conventions as the reference: errors are printed to
 * stderr, the work runs on the legacy default stream and the call ends with
 * cudaDeviceSynchronize(). */

/* reference src/kernels/flash_attention_forward.cu:795-817 */
void launch_flash_attention_forward(const void* Q, const void* K, const void* V, void* O,
                                    int batch, int heads, int seq_len, int head_dim, float scale,
                                    bool causal);
/* reference src/kernels/flash_attention_forward.cu:819-833 (d=64 only) */
void launch_flash_attention_forward_scalar(const void* Q, const void* K, const void* V, void* O,
                                           int batch, int heads, int seq_len, int head_dim,
                                           float scale, bool causal);
/* reference src/kernels/flash_attention_forward.cu:835-849 (d=64 only) */
void launch_flash_attention_forward_wmma_qk(const void* Q, const void* K, const void* V, void* O,
                                            int batch, int heads, int seq_len, int head_dim,
                                            float scale, bool causal);
/* reference src/kernels/naive_attention.cu:115-164; workspace holds
 * batch*heads*seq_len*seq_len floats (the materialised score matrix). */
void launch_naive_attention(const void* Q, const void* K, const void* V, void* O, int batch,
                            int heads, int seq_len, int head_dim, float scale, bool causal,
                            float* workspace);

/* Stream-ordered form of launch_naive_attention used by the Python binding
 * (same math, no device synchronisation, returns a status code). */
int fa_naive_fwd(const void* Q, const void* K, const void* V, void* O, int batch, int heads,
                 int seq_len, int head_dim, float scale, int causal, float* workspace,
                 void* stream);

/* fa_naive_fwd_noalloc — the materialised attention of fa_naive_fwd for
 * callers that cannot allocate device memory while they run: hosts whose
 * allocator is closed after start-up, real-time or embedded loops, runtimes
 * that own all device memory and forbid cudaMalloc from libraries.  It has no
 * counterpart in the reference (the reference's binding allocates the
 * workspace with torch::empty per call, pytorch_extension.cpp:37-40).
 *   - The score workspace is a file-scope device array of 4Mi floats
 *     (16 MiB), so batch*heads*seq_len*seq_len must be <= 4194304; larger
 *     problems return FA_ERR_SCRATCH_LIMIT and launch nothing.  Every GPU that
 *     loads this library holds those 16 MiB until the process exits.
 *   - Nothing is allocated or freed: no cudaMalloc/cudaFree, no allocating
 *     library call.  Every call looks up the array's device address
 *     (cudaGetSymbolAddress) for the calling thread's current device, so the
 *     address stays right after a cudaDeviceReset; the first call on a device
 *     may also load this library's module there, so make that first call
 *     before any stream capture on the device.
 *   - All calls on a device share the one array and it keeps the last call's
 *     contents (every score is rewritten before it is read, so nothing needs
 *     clearing).  Calls whose work overlaps on the GPU race on the array:
 *     order them on one stream or synchronise between them.
 * Arguments, layout (fp16), stream semantics and results as fa_naive_fwd. */
int fa_naive_fwd_noalloc(const void* Q, const void* K, const void* V, void* O, int batch,
                         int heads, int seq_len, int head_dim, float scale, int causal,
                         void* stream);

/* ---- standalone-kernel launchers ----
 * reference flash-attention-sm75-fused/src/flash_mha_flatargs.cu:231-252
 * (full attention, d = 64).  Asynchronous on `stream`. */
int flatargs_launch(const void* Q, const void* K, const void* V, void* O, int B, int H, int N,
                    float scale, void* stream);
/* reference flash-attention-sm75-fused/src/flash_mha_v2.cu:366-392
 * (d = 64; mode 0 = FULL, 1 = CAUSAL).  Asynchronous on `stream`. */
int launch_v2(const void* Q, const void* K, const void* V, void* O, int B, int H, int N,
              float scale, int mode, void* stream);

/* ---- diagnostics ---- */
/* Error code recorded by the device watchdog on the current device (0 if
 * none); `reset` clears it.  Synchronous (reads device memory). */
int fa_device_status(int reset);
/* Watchdog deadline for every in-kernel wait, in ns (default 1e9). */
void fa_set_watchdog_ns(unsigned long long ns);
/* FA_DEBUG_* bits applied to subsequent launches (tests only; default 0). */
void fa_set_debug_flags(int flags);
/* Development hook: device buffer (8*64*32 int64) that builds compiled with
 * FA_TRACE fill with per-tile clock64() samples; NULL disables.  No effect in
 * regular builds. */
void fa_set_trace_buffer(void* buf);
/* Human-readable text for a status code. */
const char* fa_error_string(int code);
/* Dynamic shared memory one CTA of the kernel uses for this head_dim. */
int fa_smem_bytes(int head_dim);
/* Library version string. */
const char* fa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H */
