"""HuggingFace / Llama SDPA monkey-patch (reference examples/llama_attention_replacement.py).

``apply_patch()`` rebinds ``torch.nn.functional.scaled_dot_product_attention``
to ``_patched_sdpa``, which sends eligible calls to
``flash_attention_sm75.flash_attention_forward`` and everything else, with the
arguments untouched, to the original function.  ``patch_stats()`` reports how
many calls took each path and why calls fell back.

Eligibility follows the reference (llama_attention_replacement.py:50-65), in
the same order and with the same fallback reason names:
``not_cuda``, ``not_fp16``, ``not_4d``, ``head_dim_unsupported``, ``dropout``,
``has_attn_mask``, ``kvcache_decode``.  Differences: bf16 queries are also
eligible (``not_fp16`` then means "neither fp16 nor bf16"); GQA calls (K/V with
fewer heads, HF's ``enable_gqa=True``) go to the kernel's native head mapping;
a head count that does not divide falls back with ``gqa_heads``.  Calls with a
query shorter than the keys (KV-cache decode, chunked prefill) are served by
``flash_attention_forward_kvcache`` with SDPA's own causal rule for that case
(top-left: query i sees keys j <= i); ``apply_patch(kvcache=False)`` restores
the reference behaviour of sending them to SDPA with reason ``kvcache_decode``.

Masked calls (``attn_mask`` given) whose mask is a padded batch's — per batch
entry, every query row sees one interval of keys, [k_start, k_end) cut by a
full, top-left or bottom-right causal rule — go to
``flash_attention_forward_padded`` (boolean masks, or additive masks holding
only 0 and -inf / the dtype's minimum).  Any other mask (biases, per-head
masks, holes) keeps the reference's ``has_attn_mask`` fallback, as does
``apply_patch(masks=False)``.  Query rows whose mask row is empty (padding
queries) come back as zeros, as from SDPA's CPU path; SDPA's CUDA kernels
leave implementation-defined values there, which callers discard.

Training: when autograd needs gradients of the inputs, square calls go to
``flash_attention`` / ``flash_attention_padded`` (forward and backward kernels;
the reference's patch raised in backward), and Nq != Nk calls fall back to
SDPA with reason ``requires_grad`` (the KV-cache kernel has no backward).
"""
import torch
import torch.nn.functional as F

from .ops import (flash_attention, flash_attention_forward, flash_attention_forward_kvcache,
                  flash_attention_forward_padded, flash_attention_padded)

_original_sdpa = F.scaled_dot_product_attention
_patch_active = False
_route_kvcache = True
_route_masks = True

_stats = {
    "total": 0,
    "flash": 0,
    "flash_kvcache": 0,
    "flash_masked": 0,
    "flash_autograd": 0,
    "fallback": 0,
    "fallback_reasons": {},
}

# (mask identity) -> padded-batch description or None; one model forward passes
# the same mask tensor to every layer, so it is analysed once.
_mask_cache = {"key": None, "value": None}


def _mask_key(m):
    return (m.data_ptr(), tuple(m.shape), tuple(m.stride()), m.dtype, m.device, m._version)


def padded_structure(attn_mask, B, Nq, Nk):
    """Per-entry row ranges and causal mode of a padded batch's SDPA mask.

    Returns ``(mode, q_start, q_end, k_start, k_end)`` (mode 0 full, 1
    bottom-right, 2 top-left; int32 device tensors of B entries) when every
    query row of entry b attends exactly the keys [k_start[b], hi) with hi =
    k_end[b] (full) or min(k_end[b], i + off + 1) (causal, off = Nk - Nq or 0),
    rows outside [q_start[b], q_end[b]) attending none; else None.  One host
    synchronisation.
    """
    m = attn_mask
    if m.dim() != 4 or m.size(1) != 1 or m.size(2) != Nq or m.size(3) != Nk or \
            m.size(0) not in (1, B):
        return None
    if m.dtype == torch.bool:
        keep = m[:, 0]
    elif m.is_floating_point():
        blocked = m[:, 0] <= torch.finfo(m.dtype).min
        if not bool(((m[:, 0] == 0) | blocked).all()):
            return None  # a bias, not a mask
        keep = ~blocked
    else:
        return None
    keep = keep.expand(B, Nq, Nk)
    ki = keep.to(torch.int8)
    cnt = ki.sum(-1, dtype=torch.int32)                          # [B, Nq]
    first = ki.argmax(-1).to(torch.int32)                        # first kept key
    last = (Nk - 1) - ki.flip(-1).argmax(-1).to(torch.int32)     # last kept key
    has = cnt > 0
    rows = torch.arange(Nq, device=m.device, dtype=torch.int32)
    q_start = torch.where(has, rows, Nq).amin(-1)
    q_end = torch.where(has, rows + 1, 0).amax(-1)
    k_start = torch.where(has, first, Nk).amin(-1)
    k_end = torch.where(has, last + 1, 0).amax(-1)
    empty = q_end == 0
    q_start = torch.where(empty, 0, q_start)
    k_start = torch.where(empty, 0, k_start)
    k_end = torch.where(empty, 0, k_end)
    interval = (~has) | (cnt == last - first + 1)
    in_q = (rows[None, :] >= q_start[:, None]) & (rows[None, :] < q_end[:, None])
    ok_modes = []
    for mode, off in ((0, None), (2, 0), (1, Nk - Nq)):
        hi = k_end[:, None].expand(B, Nq) if off is None else \
            torch.minimum(k_end[:, None], rows[None, :] + off + 1)
        want = in_q & (hi > k_start[:, None])
        match = (has == want) & (~has | ((first == k_start[:, None]) & (last + 1 == hi)))
        ok_modes.append((match & interval).all())
    flags = torch.stack(ok_modes).cpu()  # the one synchronisation
    for (mode, _), ok in zip(((0, None), (2, 0), (1, Nk - Nq)), flags.tolist()):
        if ok:
            return mode, q_start.int(), q_end.int(), k_start.int(), k_end.int()
    return None


def _padded_for(attn_mask, B, Nq, Nk):
    key = _mask_key(attn_mask) + (B, Nq, Nk)
    if _mask_cache["key"] != key:
        _mask_cache["value"] = padded_structure(attn_mask, B, Nq, Nk)
        _mask_cache["key"] = key
    return _mask_cache["value"]


def _record_fallback(reason: str):
    _stats["fallback"] += 1
    _stats["fallback_reasons"][reason] = _stats["fallback_reasons"].get(reason, 0) + 1


def _ineligible_reason(query, key, value, dropout_p, attn_mask, is_causal=False):
    if not query.is_cuda:
        return "not_cuda"
    if query.dtype not in (torch.float16, torch.bfloat16):
        return "not_fp16"
    if query.dim() != 4:
        return "not_4d"
    if query.size(-1) not in (64, 128):
        return "head_dim_unsupported"
    if dropout_p != 0.0:
        return "dropout"
    if attn_mask is not None and (not _route_masks or is_causal):
        return "has_attn_mask"
    if query.size(2) != key.size(2) and not _route_kvcache:
        # KV-cache decode / chunked prefill: Q is shorter than K
        return "kvcache_decode"
    if key.dim() != 4 or key.size(1) == 0 or query.size(1) % key.size(1) != 0:
        return "gqa_heads"
    if key.dtype != query.dtype or key.size(-1) != query.size(-1):
        return "not_fp16"
    if value.dim() != 4 or value.shape != key.shape or value.dtype != key.dtype:
        return "not_fp16"
    if attn_mask is not None and not (
            isinstance(attn_mask, torch.Tensor) and attn_mask.is_cuda and
            attn_mask.device == query.device and
            _padded_for(attn_mask, query.size(0), query.size(2), key.size(2)) is not None):
        return "has_attn_mask"
    if _needs_grad(query, key, value) and query.size(2) != key.size(2):
        return "requires_grad"  # the KV-cache kernel has no backward
    return None


def _needs_grad(*ts):
    return torch.is_grad_enabled() and any(getattr(t, "requires_grad", False) for t in ts)


def _patched_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                  **kwargs):
    _stats["total"] += 1
    reason = _ineligible_reason(query, key, value, dropout_p, attn_mask, is_causal)
    if reason is not None:
        _record_fallback(reason)
        return _original_sdpa(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                              is_causal=is_causal, scale=scale, **kwargs)
    _stats["flash"] += 1
    if attn_mask is not None:
        _stats["flash_masked"] += 1
        mode, qs, qe, ks, ke = _padded_for(attn_mask, query.size(0), query.size(2), key.size(2))
        if _needs_grad(query, key, value):  # square here (Nq != Nk fell back above)
            _stats["flash_autograd"] += 1
            return flash_attention_padded(query, key, value, qs, qe, ks, ke, causal=mode != 0,
                                          scale=scale)
        return flash_attention_forward_padded(
            query, key, value, qs, qe, ks, ke, causal=mode != 0, scale=scale,
            causal_alignment="top_left" if mode == 2 else "bottom_right")
    if query.size(2) != key.size(2):
        _stats["flash_kvcache"] += 1
        return flash_attention_forward_kvcache(query, key, value, causal=is_causal, scale=scale,
                                               causal_alignment="top_left")
    if _needs_grad(query, key, value):
        _stats["flash_autograd"] += 1  # training: forward + backward kernels
        return flash_attention(query, key, value, causal=is_causal, scale=scale)
    return flash_attention_forward(query, key, value, causal=is_causal, scale=scale)


def apply_patch(kvcache: bool = True, masks: bool = True):
    """Patch SDPA; ``kvcache=False`` keeps Nq != Nk calls and ``masks=False``
    masked calls on the original SDPA."""
    global _patch_active, _route_kvcache, _route_masks
    _route_kvcache = bool(kvcache)
    _route_masks = bool(masks)
    if _patch_active:
        return
    import torch.nn.functional as _F
    _F.scaled_dot_product_attention = _patched_sdpa
    torch.nn.functional.scaled_dot_product_attention = _patched_sdpa
    _patch_active = True
    print("[flash-attention-sm75] Patch applied.")


def remove_patch():
    global _patch_active
    import torch.nn.functional as _F
    _F.scaled_dot_product_attention = _original_sdpa
    torch.nn.functional.scaled_dot_product_attention = _original_sdpa
    _patch_active = False
    print("[flash-attention-sm75] Patch removed.")


def patch_stats():
    return dict(_stats, active=_patch_active)


def reset_stats():
    _stats["total"] = 0
    _stats["flash"] = 0
    _stats["flash_kvcache"] = 0
    _stats["flash_masked"] = 0
    _stats["flash_autograd"] = 0
    _stats["fallback"] = 0
    _stats["fallback_reasons"].clear()


def run_generation_test(model_name: str = "Qwen/Qwen2-0.5B-Instruct", n_new: int = 64):
    """Greedy generation with and without the patch (reference
    llama_attention_replacement.py:120-205); needs the model weights locally."""
    import time

    from transformers import AutoModelForCausalLM, AutoTokenizer

    tokenizer = AutoTokenizer.from_pretrained(model_name)
    model = AutoModelForCausalLM.from_pretrained(model_name, torch_dtype=torch.float16,
                                                 device_map="cuda", attn_implementation="sdpa")
    model.eval()
    inputs = tokenizer("The key insight of FlashAttention is", return_tensors="pt").to("cuda")
    with torch.no_grad():
        t0 = time.perf_counter()
        ref = model.generate(**inputs, max_new_tokens=n_new, do_sample=False)
        t_ref = time.perf_counter() - t0
    apply_patch()
    reset_stats()
    try:
        with torch.no_grad():
            t0 = time.perf_counter()
            out = model.generate(**inputs, max_new_tokens=n_new, do_sample=False)
            t_pat = time.perf_counter() - t0
    finally:
        remove_patch()
    return {
        "text_ref": tokenizer.decode(ref[0], skip_special_tokens=True),
        "text_patched": tokenizer.decode(out[0], skip_special_tokens=True),
        "identical": bool(torch.equal(ref, out)),
        "ms_ref": t_ref * 1e3, "ms_patched": t_pat * 1e3, "stats": patch_stats(),
    }
