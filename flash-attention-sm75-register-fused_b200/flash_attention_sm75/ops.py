"""Python entry point of the attention forward (reference src/flash_attention_sm75/ops.py).

``flash_attention_forward(Q, K, V, causal=False, scale=None)`` keeps the
reference's signature, argument checks and error types:

* ``ValueError`` if Q is not 4-D (ops.py:70-71);
* ``RuntimeError`` containing "supports head_dim=64 or 128" (ops.py:74-77);
* ``RuntimeError`` "GQA expansion: Q heads (..) not divisible by K/V heads (..)"
  (ops.py:19-22);
* backward raises ``NotImplementedError`` (ops.py:47-52).

Differences that a caller can observe only as speed or as extra options:

* GQA/MQA is served natively: query head ``h`` reads KV head ``h // (Hq/Hkv)``
  inside the kernel — the same mapping as the reference's ``repeat_interleave``
  expansion (ops.py:24-26) — so K/V are never copied.
* bf16 inputs are accepted in addition to fp16.
* ``return_lse=True`` also returns the fp32 log-sum-exp ``[B, Hq, N]``.
* ``flash_attention_forward_kvcache`` (no reference counterpart) serves
  ``Nq != Nk`` — KV-cache decode and chunked prefill — with bottom-right or
  top-left causal alignment.
* ``flash_attention_forward_host`` takes Q, K, V in host memory and returns O
  in host memory, overlapping the PCIe copies of each (batch, KV-head group)
  chunk with the computation of the others.
* ``flash_attention`` is the same forward with a backward pass (dQ, dK, dV
  from the saved LSE); ``flash_attention_forward`` keeps the reference's
  forward-only Function.

There is no CPU path: the CUDA extension must load, or the import fails.
"""
import math

import torch

import flash_attn_sm75_cuda as _C


def _expand_kv_for_gqa(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor):
    """Reference-compatible helper (ops.py:6-27): K/V repeated to Q's head count.

    Kept for callers that import it; ``flash_attention_forward`` itself does
    not use it, because the kernel maps heads without copying.
    """
    h_q = Q.size(1)
    h_kv = K.size(1)
    if h_q == h_kv:
        return K, V
    _check_gqa(h_q, h_kv)
    factor = h_q // h_kv
    K = K.repeat_interleave(factor, dim=1).contiguous()
    V = V.repeat_interleave(factor, dim=1).contiguous()
    return K, V


def _check_gqa(h_q: int, h_kv: int) -> None:
    if h_kv == 0 or h_q % h_kv != 0:
        raise RuntimeError(
            f"GQA expansion: Q heads ({h_q}) not divisible by K/V heads ({h_kv})"
        )


class FlashAttentionSM75Function(torch.autograd.Function):
    """Autograd wrapper (reference ops.py:30-52); forward only."""

    @staticmethod
    def forward(ctx, Q, K, V, causal, scale, return_lse=False):
        _check_gqa(Q.size(1), K.size(1))
        Q = Q.contiguous()
        K = K.contiguous()
        V = V.contiguous()
        if return_lse:
            out, lse = _C.flash_attention_forward_lse(Q, K, V, bool(causal), float(scale))
            ctx.mark_non_differentiable(lse)
            ctx.save_for_backward(Q, K, V, out)
            return out, lse
        out = _C.flash_attention_forward(Q, K, V, bool(causal), float(scale))
        ctx.save_for_backward(Q, K, V, out)
        return out

    @staticmethod
    def backward(ctx, *grad_outputs):
        raise NotImplementedError(
            "Backward pass not implemented. "
            "flash-attention-sm75 is for inference only "
            "(Backward pass is not implemented for this forward-only kernel)."
        )


def flash_attention_forward(Q, K, V, causal=False, scale=None, return_lse=False):
    """Drop-in for ``F.scaled_dot_product_attention`` (forward) on B200.

    Args:
        Q: [B, H_q,  N, D]  float16 / bfloat16, cuda
        K: [B, H_kv, N, D]  same dtype, H_kv divides H_q
        V: [B, H_kv, N, D]  same dtype
        causal: bool — top-left causal mask (query i sees keys j <= i)
        scale:  float (default 1/sqrt(D))
        return_lse: also return LSE [B, H_q, N] fp32 (natural log)

    Returns:
        O: [B, H_q, N, D] (and LSE when ``return_lse``)
    """
    if Q.dim() != 4:
        raise ValueError("Q must be 4D [B, H, N, D]")

    head_dim = Q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )

    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)

    return FlashAttentionSM75Function.apply(Q, K, V, causal, scale, return_lse)


_CAUSAL_MODES = {"bottom_right": 1, "top_left": 2}


def flash_attention_forward_kvcache(Q, K, V, causal=False, scale=None, return_lse=False,
                                    causal_alignment="bottom_right"):
    """Attention of ``Nq`` new queries against ``Nk`` cached keys (decode,
    chunked prefill); forward only.

    Args:
        Q: [B, H_q,  N_q, D]  float16 / bfloat16, cuda
        K: [B, H_kv, N_k, D]  same dtype, H_kv divides H_q
        V: [B, H_kv, N_k, D]  same dtype
        causal: bool
        scale: float (default 1/sqrt(D))
        return_lse: also return LSE [B, H_q, N_q] fp32 (natural log)
        causal_alignment: "bottom_right" (query i sees keys j <= i + N_k - N_q,
            the KV-cache convention) or "top_left" (j <= i, the rule of
            ``F.scaled_dot_product_attention(is_causal=True)`` for N_q != N_k)

    Rows that see no key (bottom-right with N_q > N_k) return O = 0, LSE = -inf.
    """
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise ValueError("Q, K, V must be 4D [B, H, N, D]")
    head_dim = Q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    if causal and causal_alignment not in _CAUSAL_MODES:
        raise ValueError(f"causal_alignment must be one of {sorted(_CAUSAL_MODES)}")
    _check_gqa(Q.size(1), K.size(1))
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    mode = _CAUSAL_MODES[causal_alignment] if causal else 0
    out, lse = _C.flash_attention_forward_kvcache(Q.contiguous(), K.contiguous(), V.contiguous(),
                                                  mode, float(scale))
    return (out, lse) if return_lse else out


def _rows_tensor(x, n, device, name):
    """int32 device tensor of n row offsets from a tensor or a sequence of ints."""
    t = torch.as_tensor(x, dtype=torch.int32, device=device).contiguous()
    if t.dim() != 1 or t.numel() != n:
        raise ValueError(f"{name} must hold {n} row offsets, got shape {tuple(t.shape)}")
    return t


def flash_attention_varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                   max_seqlen_k, causal=False, scale=None, return_lse=False,
                                   causal_alignment="bottom_right"):
    """Attention over a packed batch of variable-length sequences; forward only.

    Args:
        q: [total_q, H_q, D]  float16 / bfloat16, cuda (sequences one after another)
        k, v: [total_k, H_kv, D]  same dtype, H_kv divides H_q
        cu_seqlens_q, cu_seqlens_k: B + 1 row offsets (int32 tensor or ints);
            sequence b owns rows [cu[b], cu[b+1])
        max_seqlen_q, max_seqlen_k: upper bounds of the sequence lengths
        causal: bool; causal_alignment "bottom_right" (query i of a sequence
            sees keys j <= i + n_k - n_q) or "top_left" (j <= i)
        scale: float (default 1/sqrt(D))
        return_lse: also return LSE [H_q, total_q] fp32 (natural log)

    Rows that see no key (and rows outside every sequence) return O = 0,
    LSE = -inf.
    """
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be 3D [total, H, D]")
    head_dim = q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    if causal and causal_alignment not in _CAUSAL_MODES:
        raise ValueError(f"causal_alignment must be one of {sorted(_CAUSAL_MODES)}")
    _check_gqa(q.size(1), k.size(1))
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    cu_q = torch.as_tensor(cu_seqlens_q, dtype=torch.int32, device=q.device).contiguous()
    cu_k = _rows_tensor(cu_seqlens_k, cu_q.numel(), q.device, "cu_seqlens_k")
    mode = _CAUSAL_MODES[causal_alignment] if causal else 0
    out, lse = _C.flash_attention_forward_varlen(q.contiguous(), k.contiguous(), v.contiguous(),
                                                 cu_q, cu_k, int(max_seqlen_q),
                                                 int(max_seqlen_k), mode, float(scale))
    return (out, lse) if return_lse else out


def flash_attention_forward_padded(Q, K, V, q_start, q_end, k_start, k_end, causal=False,
                                   scale=None, return_lse=False, causal_alignment="bottom_right"):
    """Attention of a padded batch without repacking; forward only.

    Args:
        Q: [B, H_q, N_q, D], K/V: [B, H_kv, N_k, D] (as ``flash_attention_forward_kvcache``)
        q_start, q_end: per batch entry, valid query rows [q_start[b], q_end[b])
        k_start, k_end: per batch entry, valid key rows [k_start[b], k_end[b])
            (int32 tensors or sequences of B ints; left padding: start > 0,
            right padding: end < N)
        causal, causal_alignment: the causal rule of the full padded rows
            ("bottom_right": key j visible to query i iff j <= i + N_k - N_q;
            "top_left": j <= i), restricted to the valid keys

    Padding keys are never attended.  Rows outside a query range, and rows
    that see no key, return O = 0, LSE = -inf.
    """
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise ValueError("Q, K, V must be 4D [B, H, N, D]")
    head_dim = Q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    if causal and causal_alignment not in _CAUSAL_MODES:
        raise ValueError(f"causal_alignment must be one of {sorted(_CAUSAL_MODES)}")
    _check_gqa(Q.size(1), K.size(1))
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    B = Q.size(0)
    ranges = [_rows_tensor(x, B, Q.device, name) for x, name in
              ((q_start, "q_start"), (q_end, "q_end"), (k_start, "k_start"), (k_end, "k_end"))]
    mode = _CAUSAL_MODES[causal_alignment] if causal else 0
    out, lse = _C.flash_attention_forward_padded(Q.contiguous(), K.contiguous(), V.contiguous(),
                                                 *ranges, mode, float(scale))
    return (out, lse) if return_lse else out


class FlashAttentionPaddedFunction(torch.autograd.Function):
    """Padded-batch attention with forward and backward (square N)."""

    @staticmethod
    def forward(ctx, Q, K, V, q_start, q_end, k_start, k_end, causal, scale):
        _check_gqa(Q.size(1), K.size(1))
        Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
        out, lse = _C.flash_attention_forward_padded(Q, K, V, q_start, q_end, k_start, k_end,
                                                     1 if causal else 0, float(scale))
        ctx.save_for_backward(Q, K, V, out, lse, q_start, q_end, k_start, k_end)
        ctx.causal, ctx.scale = bool(causal), float(scale)
        return out

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, out, lse, qs, qe, ks, ke = ctx.saved_tensors
        dQ, dK, dV = _C.flash_attention_backward_padded(dO.contiguous(), Q, K, V, out, lse, qs, qe,
                                                        ks, ke, ctx.causal, ctx.scale)
        return dQ, dK, dV, None, None, None, None, None, None


def flash_attention_padded(Q, K, V, q_start, q_end, k_start, k_end, causal=False, scale=None):
    """``flash_attention_forward_padded`` with autograd support for square
    padded batches (Q, K, V all [B, H, N, D]): padding keys get zero dK / dV,
    query rows outside the ranges zero dQ."""
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise ValueError("Q, K, V must be 4D [B, H, N, D]")
    if Q.size(2) != K.size(2):
        raise ValueError("flash_attention_padded needs Nq == Nk")
    head_dim = Q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    B = Q.size(0)
    ranges = [_rows_tensor(x, B, Q.device, name) for x, name in
              ((q_start, "q_start"), (q_end, "q_end"), (k_start, "k_start"), (k_end, "k_end"))]
    return FlashAttentionPaddedFunction.apply(Q, K, V, *ranges, causal, scale)


class FlashAttentionVarlenFunction(torch.autograd.Function):
    """Packed variable-length self-attention with forward and backward."""

    @staticmethod
    def forward(ctx, q, k, v, cu, max_seqlen, causal, scale):
        _check_gqa(q.size(1), k.size(1))
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        out, lse = _C.flash_attention_forward_varlen(q, k, v, cu, cu, int(max_seqlen),
                                                     int(max_seqlen), 1 if causal else 0,
                                                     float(scale))
        ctx.save_for_backward(q, k, v, out, lse, cu)
        ctx.max_seqlen, ctx.causal, ctx.scale = int(max_seqlen), bool(causal), float(scale)
        return out

    @staticmethod
    def backward(ctx, dO):
        q, k, v, out, lse, cu = ctx.saved_tensors
        dq, dk, dv = _C.flash_attention_backward_varlen(dO.contiguous(), q, k, v, out, lse, cu,
                                                        ctx.max_seqlen, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None, None, None


def flash_attention_varlen(q, k, v, cu_seqlens, max_seqlen, causal=False, scale=None):
    """``flash_attention_varlen_forward`` with autograd support for packed
    self-attention batches (one ``cu_seqlens`` for queries and keys): q
    [total, H_q, D], k / v [total, H_kv, D]."""
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("q, k, v must be 3D [total, H, D]")
    if q.size(0) != k.size(0):
        raise ValueError("flash_attention_varlen is self-attention: q and k share their rows")
    head_dim = q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    cu = torch.as_tensor(cu_seqlens, dtype=torch.int32, device=q.device).contiguous()
    return FlashAttentionVarlenFunction.apply(q, k, v, cu, max_seqlen, causal, scale)


_pipeline = {}


def _pipeline_streams(index):
    if index not in _pipeline:
        _pipeline[index] = tuple(torch.cuda.Stream(device=index) for _ in range(3))
    return _pipeline[index]


def _halving_slices(units, max_slices):
    """Slice sizes (in units) for the host pipeline: each slice takes half of
    the units that remain (the last of ``max_slices`` takes them all)."""
    sizes, rem = [], units
    while rem > 0:
        n = rem if len(sizes) == max_slices - 1 else (rem + 1) // 2
        sizes.append(n)
        rem -= n
    return sizes


def flash_attention_forward_host(Q, K, V, causal=False, scale=None, out=None, device=None,
                                 chunks=32):
    """Attention forward of host-resident Q, K, V into host-resident O.

    The work is cut into at most ``chunks`` slices of whole KV-head groups,
    counted over the flattened (batch, KV head) index, which is contiguous in
    all four tensors.  Each slice takes half of the groups that remain, so
    the copies are few and large while the last slices, whose forward and
    copy back run after the last input copy, are small.  Per slice, Q/K/V are
    copied to the GPU on a copy stream, the forward runs on a compute stream
    once they have landed, and O is copied back on a third stream, so
    transfers in both directions overlap the computation of other slices (use
    pinned host tensors for asynchronous copies).  Measured on B200 for C5
    (805 MB in): 16.1 ms per call against 17.1 ms with 32 equal slices and a
    15.5 ms floor for the same copies alone.  Returns ``out`` (allocated
    pinned if None) once it holds the result.
    """
    if Q.dim() != 4 or K.dim() != 4 or V.dim() != 4:
        raise ValueError("Q must be 4D [B, H, N, D]")
    if Q.is_cuda or K.is_cuda or V.is_cuda:
        raise ValueError("flash_attention_forward_host expects host tensors")
    head_dim = Q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    _check_gqa(Q.size(1), K.size(1))
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
    B, Hq, N, _ = Q.shape
    Hkv = K.size(1)
    G = Hq // Hkv
    if out is None:
        out = torch.empty(Q.shape, dtype=Q.dtype, pin_memory=True)
    if out.shape != Q.shape or out.dtype != Q.dtype or not out.is_contiguous() or out.is_cuda:
        raise ValueError("out must be a contiguous host tensor shaped and typed like Q")
    if Q.numel() == 0:
        return out
    dev = torch.device("cuda", torch.cuda.current_device() if device is None
                       else torch.device(device).index)
    # [B*H, N, d] views: a run of (batch, head) units is one contiguous block
    q3, k3, v3 = (t.view(-1, N, head_dim) for t in (Q, K, V))
    o3 = out.view(-1, N, head_dim)
    sizes = _halving_slices(B * Hkv, max(1, int(chunks)))
    with torch.cuda.device(dev):
        cur = torch.cuda.current_stream()
        s_in, s_comp, s_out = _pipeline_streams(dev.index)
        dq = torch.empty(q3.shape, dtype=Q.dtype, device=dev)
        dk = torch.empty(k3.shape, dtype=K.dtype, device=dev)
        dv = torch.empty(v3.shape, dtype=V.dtype, device=dev)
        do = torch.empty(q3.shape, dtype=Q.dtype, device=dev)
        for t, st in ((dq, s_in), (dk, s_in), (dv, s_in), (dq, s_comp), (dk, s_comp),
                      (dv, s_comp), (do, s_comp), (do, s_out)):
            t.record_stream(st)
        for st in (s_in, s_comp, s_out):
            st.wait_stream(cur)
        u0 = 0
        for n in sizes:
            u1 = u0 + n
            h0, h1 = u0 * G, u1 * G
            with torch.cuda.stream(s_in):
                dq[h0:h1].copy_(q3[h0:h1], non_blocking=True)
                dk[u0:u1].copy_(k3[u0:u1], non_blocking=True)
                dv[u0:u1].copy_(v3[u0:u1], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(landed)
                # a slice is one batch entry of its units' heads
                _C.flash_attention_forward_out(dq[h0:h1].unsqueeze(0), dk[u0:u1].unsqueeze(0),
                                               dv[u0:u1].unsqueeze(0), do[h0:h1].unsqueeze(0),
                                               None, bool(causal), float(scale))
                done = torch.cuda.Event()
                done.record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                o3[h0:h1].copy_(do[h0:h1], non_blocking=True)
            u0 = u1
        cur.wait_stream(s_out)
        s_out.synchronize()
    return out


class FlashAttentionFunction(torch.autograd.Function):
    """Forward and backward (no reference counterpart: the reference's Function
    raises in backward, ops.py:47-52)."""

    @staticmethod
    def forward(ctx, Q, K, V, causal, scale):
        _check_gqa(Q.size(1), K.size(1))
        Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
        out, lse = _C.flash_attention_forward_lse(Q, K, V, bool(causal), float(scale))
        ctx.save_for_backward(Q, K, V, out, lse)
        ctx.causal, ctx.scale = bool(causal), float(scale)
        return out

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, out, lse = ctx.saved_tensors
        dQ, dK, dV = _C.flash_attention_backward(dO.contiguous(), Q, K, V, out, lse, ctx.causal,
                                                 ctx.scale)
        return dQ, dK, dV, None, None


def flash_attention(Q, K, V, causal=False, scale=None):
    """``flash_attention_forward`` with autograd support (dQ, dK, dV on the GPU).

    Same arguments and checks as ``flash_attention_forward`` (Q [B, Hq, N, D],
    K/V [B, Hkv, N, D], D in {64, 128}, fp16/bf16, top-left causal).
    """
    if Q.dim() != 4:
        raise ValueError("Q must be 4D [B, H, N, D]")
    head_dim = Q.size(-1)
    if head_dim not in (64, 128):
        raise RuntimeError(
            f"flash_attention_sm75 supports head_dim=64 or 128, got {head_dim}"
        )
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    return FlashAttentionFunction.apply(Q, K, V, causal, scale)
