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


def test_padded_mask_structure_cpu():
    """The mask analysis that routes masked calls to the padded kernel (CPU
    tensors; the routing itself needs CUDA tensors)."""
    from tests.test_varlen_cpu import padded_mask
    B, N = 3, 40
    qr = [(0, 40), (7, 40), (0, 25)]
    kr = [(0, 40), (7, 40), (0, 25)]
    for mode in (0, 1, 2):
        m = padded_mask(B, N, N, qr, kr, mode)
        got = patch.padded_structure(m, B, N, N)
        assert got is not None
        want_mode = 0 if mode == 0 else 2  # square: top-left and bottom-right coincide
        assert got[0] == want_mode
        assert got[1].tolist() == [0, 7, 0] and got[2].tolist() == [40, 40, 25]
        assert got[3].tolist() == [0, 7, 0] and got[4].tolist() == [40, 40, 25]
        # the additive form of the same mask
        add = torch.zeros(m.shape).masked_fill(~m, torch.finfo(torch.float32).min)
        assert patch.padded_structure(add, B, N, N)[0] == want_mode
    # decode over a left-padded cache: one query row, keys [pad, Nk)
    m = padded_mask(2, 1, 50, [(0, 1), (0, 1)], [(10, 50), (0, 50)], 1)
    got = patch.padded_structure(m, 2, 1, 50)
    assert got is not None and got[3].tolist() == [10, 0] and got[4].tolist() == [50, 50]
    # holes, biases and per-head masks are not padded batches
    m = padded_mask(B, N, N, qr, kr, 1)
    m[1, 0, 20, 10] = False
    assert patch.padded_structure(m, B, N, N) is None
    bias = torch.randn(1, 1, N, N)
    assert patch.padded_structure(bias, 1, N, N) is None
    assert patch.padded_structure(torch.ones(1, 2, N, N, dtype=torch.bool), 1, N, N) is None


def test_requires_grad_routing_cpu():
    """Calls that need gradients: Nq != Nk ones fall back with reason
    requires_grad (checked on fake CUDA tensors; the routing of square calls
    to the autograd kernels is tested on the GPU)."""
    class Fake:
        def __init__(self, shape=(1, 2, 8, 64), grad=True):
            self.is_cuda, self.dtype, self._s = True, torch.float16, shape
            self.shape = torch.Size(shape)
            self.requires_grad = grad

        def dim(self):
            return len(self._s)

        def size(self, i):
            return self._s[i]

    r = patch._ineligible_reason
    q, kv = Fake((1, 2, 1, 64)), Fake((1, 2, 8, 64))
    assert r(q, kv, kv, 0.0, None) == "requires_grad"  # Nq != Nk
    with torch.no_grad():
        assert r(q, kv, kv, 0.0, None) is None
    assert r(Fake(), Fake(), Fake(), 0.0, None) is None  # square, unmasked: autograd kernels
