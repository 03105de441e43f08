"""ctypes binding of the C ABI in include/fa_b200.h.

Loads the in-tree ``lib/libfa_b200.so`` and declares every entry point with
its C signature, so Python callers (tests, bench.py, hosts without the pybind
module) call the same boundary a C or cgo host would.  Torch is used only to
obtain device pointers and the current stream in the tensor helpers.
"""
import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libfa_b200.so")

c_vp, c_int, c_float, c_bool = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_bool

SIGNATURES = {
    "fa_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_float,
                       c_int, c_int, c_vp]),
    "fa_fwd_kvcache": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_int,
                               c_int, c_float, c_int, c_int, c_vp, ctypes.c_size_t, c_vp]),
    "fa_fwd_kvcache_workspace_bytes": (ctypes.c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "fa_bwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                       c_int, c_int, c_float, c_int, c_int, c_vp, ctypes.c_size_t, c_vp]),
    "fa_bwd_workspace_bytes": (ctypes.c_size_t, [c_int, c_int, c_int]),
    "fa_bwd_padded": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                              c_vp, c_vp, c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_int,
                              c_vp, ctypes.c_size_t, c_vp]),
    "fa_bwd_varlen": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int,
                              c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_vp,
                              ctypes.c_size_t, c_vp]),
    "fa_fwd_varlen": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int,
                              c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_vp]),
    "fa_fwd_padded": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int,
                              c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_vp]),
    "launch_flash_attention_forward": (None, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int,
                                              c_float, c_bool]),
    "launch_flash_attention_forward_scalar": (None, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                                     c_int, c_float, c_bool]),
    "launch_flash_attention_forward_wmma_qk": (None, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                                      c_int, c_float, c_bool]),
    "launch_naive_attention": (None, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float,
                                      c_bool, c_vp]),
    "fa_naive_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float, c_int,
                             c_vp, c_vp]),
    "fa_naive_fwd_noalloc": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_float,
                                     c_int, c_vp]),
    "flatargs_launch": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_float, c_vp]),
    "launch_v2": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_float, c_int, c_vp]),
    "fa_device_status": (c_int, [c_int]),
    "fa_set_watchdog_ns": (None, [ctypes.c_ulonglong]),
    "fa_set_debug_flags": (None, [c_int]),
    "fa_set_trace_buffer": (None, [c_vp]),
    "fa_error_string": (ctypes.c_char_p, [c_int]),
    "fa_smem_bytes": (c_int, [c_int]),
    "fa_version": (ctypes.c_char_p, []),
}

_lib = None


def load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_ptr(torch_stream=None):
    import torch
    s = torch_stream or torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def fa_fwd(q, k, v, o, lse=None, causal=False, scale=None, stream=None):
    """Call fa_fwd on torch CUDA tensors laid out [B, H, N, d]; returns the status."""
    import math
    import torch
    B, Hq, N, d = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    return load().fa_fwd(ptr(q), ptr(k), ptr(v), ptr(o), ptr(lse), B, Hq, Hkv, N, d,
                         float(scale), int(bool(causal)), dtype, stream_ptr(stream))


CAUSAL_NONE, CAUSAL_BOTTOM_RIGHT, CAUSAL_TOP_LEFT = 0, 1, 2


def fa_fwd_kvcache(q, k, v, o, lse=None, causal=CAUSAL_NONE, scale=None, stream=None,
                   workspace=True):
    """Call fa_fwd_kvcache on torch CUDA tensors (Q/O [B, Hq, Nq, d], K/V
    [B, Hkv, Nk, d]); ``workspace=True`` allocates the split workspace the
    library asks for, ``None`` runs unsplit.  Returns the status."""
    import math
    import torch
    B, Hq, Nq, d = q.shape
    Hkv, Nk = k.shape[1], k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    lib = load()
    ws, nbytes = None, 0
    if workspace is True:
        nbytes = lib.fa_fwd_kvcache_workspace_bytes(B, Hq, Hkv, Nq, Nk, d)
        if nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    elif workspace is not None:
        ws, nbytes = workspace, workspace.numel() * workspace.element_size()
    return lib.fa_fwd_kvcache(ptr(q), ptr(k), ptr(v), ptr(o), ptr(lse), B, Hq, Hkv, Nq, Nk, d,
                              float(scale), int(causal), dtype, ptr(ws), nbytes,
                              stream_ptr(stream))


def fa_bwd(q, k, v, o, do, lse, dq, dk, dv, causal=False, scale=None, stream=None):
    """Call fa_bwd on torch CUDA tensors ([B, H, N, d]; lse [B, Hq, N] fp32);
    allocates the workspace.  Returns the status."""
    import math
    import torch
    B, Hq, N, d = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    lib = load()
    nbytes = lib.fa_bwd_workspace_bytes(B, Hq, N)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    return lib.fa_bwd(ptr(q), ptr(k), ptr(v), ptr(o), ptr(do), ptr(lse), ptr(dq), ptr(dk), ptr(dv),
                      B, Hq, Hkv, N, d, float(scale), int(bool(causal)), dtype, ptr(ws), nbytes,
                      stream_ptr(stream))


def fa_fwd_varlen(q, k, v, o, lse, cu_q, cu_k, max_q, max_k, causal=CAUSAL_NONE, scale=None,
                  stream=None):
    """Call fa_fwd_varlen on packed torch CUDA tensors (Q/O [total_q, Hq, d],
    K/V [total_k, Hkv, d], LSE [Hq, total_q] or None, cu_* int32 [B + 1] on the
    device).  Returns the status."""
    import math
    import torch
    Tq, Hq, d = q.shape
    Tk, Hkv = k.shape[0], k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    return load().fa_fwd_varlen(ptr(q), ptr(k), ptr(v), ptr(o), ptr(lse), ptr(cu_q), ptr(cu_k),
                                cu_q.numel() - 1, Hq, Hkv, Tq, Tk, int(max_q), int(max_k), d,
                                float(scale), int(causal), dtype, stream_ptr(stream))


def fa_fwd_padded(q, k, v, o, lse, q_start, q_end, k_start, k_end, causal=CAUSAL_NONE,
                  scale=None, stream=None):
    """Call fa_fwd_padded on torch CUDA tensors (Q/O [B, Hq, Nq, d], K/V
    [B, Hkv, Nk, d], LSE [B, Hq, Nq] or None, row ranges int32 [B] on the
    device).  Returns the status."""
    import math
    import torch
    B, Hq, Nq, d = q.shape
    Hkv, Nk = k.shape[1], k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    return load().fa_fwd_padded(ptr(q), ptr(k), ptr(v), ptr(o), ptr(lse), ptr(q_start),
                                ptr(q_end), ptr(k_start), ptr(k_end), B, Hq, Hkv, Nq, Nk, d,
                                float(scale), int(causal), dtype, stream_ptr(stream))


def fa_bwd_padded(q, k, v, o, do, lse, q_start, q_end, k_start, k_end, dq, dk, dv, causal=False,
                  scale=None, stream=None):
    """Call fa_bwd_padded on torch CUDA tensors ([B, H, N, d]; lse [B, Hq, N]
    fp32; row ranges int32 [B]); allocates the workspace.  Returns the status."""
    import math
    import torch
    B, Hq, N, d = q.shape
    Hkv = k.shape[1]
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    lib = load()
    nbytes = lib.fa_bwd_workspace_bytes(B, Hq, N)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    return lib.fa_bwd_padded(ptr(q), ptr(k), ptr(v), ptr(o), ptr(do), ptr(lse), ptr(q_start),
                             ptr(q_end), ptr(k_start), ptr(k_end), ptr(dq), ptr(dk), ptr(dv), B, Hq,
                             Hkv, N, d, float(scale), int(bool(causal)), dtype, ptr(ws), nbytes,
                             stream_ptr(stream))


def fa_bwd_varlen(q, k, v, o, do, lse, cu, max_seqlen, dq, dk, dv, causal=False, scale=None,
                  stream=None):
    """Call fa_bwd_varlen on packed torch CUDA tensors ([total, H, d]; lse
    [Hq, total] fp32; cu int32 [B + 1]); allocates the workspace.  Returns the
    status."""
    import math
    import torch
    T, Hq, d = q.shape
    Hkv = k.shape[1]
    B = cu.numel() - 1
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    lib = load()
    nbytes = lib.fa_bwd_workspace_bytes(B, Hq, int(max_seqlen))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    return lib.fa_bwd_varlen(ptr(q), ptr(k), ptr(v), ptr(o), ptr(do), ptr(lse), ptr(cu), ptr(dq),
                             ptr(dk), ptr(dv), B, Hq, Hkv, T, int(max_seqlen), d, float(scale),
                             int(bool(causal)), dtype, ptr(ws), nbytes, stream_ptr(stream))
