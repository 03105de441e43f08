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
"""
import torch
import torch.nn.functional as F

from .ops import flash_attention_forward, flash_attention_forward_kvcache

_original_sdpa = F.scaled_dot_product_attention
_patch_active = False
_route_kvcache = True

_stats = {
    "total": 0,
    "flash": 0,
    "flash_kvcache": 0,
    "fallback": 0,
    "fallback_reasons": {},
}


def _record_fallback(reason: str):
    _stats["fallback"] += 1
    _stats["fallback_reasons"][reason] = _stats["fallback_reasons"].get(reason, 0) + 1


def _ineligible_reason(query, key, value, dropout_p, attn_mask):
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
    if attn_mask is not None:
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
    return None


def _patched_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                  **kwargs):
    _stats["total"] += 1
    reason = _ineligible_reason(query, key, value, dropout_p, attn_mask)
    if reason is not None:
        _record_fallback(reason)
        return _original_sdpa(query, key, value, attn_mask=attn_mask, dropout_p=dropout_p,
                              is_causal=is_causal, scale=scale, **kwargs)
    _stats["flash"] += 1
    if query.size(2) != key.size(2):
        _stats["flash_kvcache"] += 1
        return flash_attention_forward_kvcache(query, key, value, causal=is_causal, scale=scale,
                                               causal_alignment="top_left")
    return flash_attention_forward(query, key, value, causal=is_causal, scale=scale)


def apply_patch(kvcache: bool = True):
    """Patch SDPA; ``kvcache=False`` keeps Nq != Nk calls on the original SDPA."""
    global _patch_active, _route_kvcache
    _route_kvcache = bool(kvcache)
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
