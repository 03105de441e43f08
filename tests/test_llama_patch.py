"""SDPA monkey-patch host logic (reference examples/llama_attention_replacement.py)
on CPU tensors: every call falls back with the reference's reason names."""
import torch
import torch.nn.functional as F

from flash_attention_sm75 import llama_attention_replacement as patch


def test_apply_remove_and_cpu_fallback():
    patch.reset_stats()
    orig = F.scaled_dot_product_attention
    patch.apply_patch()
    try:
        assert F.scaled_dot_product_attention is patch._patched_sdpa
        q = torch.randn(1, 2, 8, 64)
        out = F.scaled_dot_product_attention(q, q, q, is_causal=True)
        ref = patch._original_sdpa(q, q, q, is_causal=True)
        assert torch.equal(out, ref)
        s = patch.patch_stats()
        assert s["active"] and s["total"] == 1 and s["flash"] == 0
        assert s["fallback_reasons"] == {"not_cuda": 1}
    finally:
        patch.remove_patch()
    assert F.scaled_dot_product_attention is orig
    assert not patch.patch_stats()["active"]


def test_reason_order_matches_reference():
    class Fake:
        def __init__(self, cuda=True, dtype=torch.float16, shape=(1, 2, 8, 64)):
            self.is_cuda, self.dtype, self._s = cuda, dtype, shape
            self.shape = torch.Size(shape)

        def dim(self):
            return len(self._s)

        def size(self, i):
            return self._s[i]

    def r(q, k, dropout, mask):
        return patch._ineligible_reason(q, k, k, dropout, mask)

    assert r(Fake(cuda=False), Fake(), 0.0, None) == "not_cuda"
    assert r(Fake(dtype=torch.float32), Fake(), 0.0, None) == "not_fp16"
    assert r(Fake(shape=(2, 8, 64)), Fake(), 0.0, None) == "not_4d"
    assert r(Fake(shape=(1, 2, 8, 96)), Fake(), 0.0, None) == "head_dim_unsupported"
    assert r(Fake(), Fake(), 0.1, None) == "dropout"
    assert r(Fake(), Fake(), 0.0, object()) == "has_attn_mask"
    # Nq != Nk: served by the kv-cache kernel, or (kvcache=False) the reference's fallback
    assert r(Fake(shape=(1, 2, 1, 64)), Fake(shape=(1, 2, 8, 64)), 0.0, None) is None
    saved = patch._route_kvcache
    patch._route_kvcache = False
    try:
        assert r(Fake(shape=(1, 2, 1, 64)), Fake(shape=(1, 2, 8, 64)), 0.0, None) == "kvcache_decode"
    finally:
        patch._route_kvcache = saved
    assert r(Fake(shape=(1, 6, 8, 64)), Fake(shape=(1, 4, 8, 64)), 0.0, None) == "gqa_heads"
    assert r(Fake(), Fake(), 0.0, None) is None
    assert r(Fake(dtype=torch.bfloat16), Fake(dtype=torch.bfloat16), 0.0, None) is None
    assert r(Fake(shape=(1, 8, 8, 128)), Fake(shape=(1, 2, 8, 128)), 0.0, None) is None
