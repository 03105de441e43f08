"""Drop-in behaviour of the Python API and the pybind module on the GPU
(reference tests/test_api.py, test_flash_d128.py, test_correctness.py,
test_flash_wmma_qk*.py), checked against the CPU oracle."""
import math

import pytest
import torch
import torch.nn.functional as F

import flash_attention_sm75 as fa
import flash_attn_sm75_cuda as C
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu


def _inputs(B, Hq, Hkv, N, d, causal=False, dtype=torch.float16, seed=42):
    cfg = orc.AttnConfig("t", B, Hq, Hkv, N, d, causal)
    return orc.make_inputs(cfg, seed=seed, dtype=dtype)


@pytest.mark.parametrize("B,H,N,d,causal", [
    (1, 8, 128, 64, False), (1, 8, 512, 64, False), (1, 8, 1024, 64, True),
    (1, 8, 128, 128, False), (2, 8, 256, 128, False), (1, 16, 512, 128, False),
    (1, 8, 1024, 128, True), (2, 16, 1024, 64, False), (1, 32, 128, 64, False),
    (1, 8, 1, 64, True), (2, 8, 16, 64, True)])
def test_extension_matches_reference_allclose(sm100, B, H, N, d, causal):
    """The reference's own parity test shape list and criterion (allclose 1e-2)."""
    q, k, v = _inputs(B, H, H, N, d, causal)
    out = C.flash_attention_forward(q.cuda(), k.cuda(), v.cuda(), causal, 1.0 / math.sqrt(d))
    ref = orc.attention_reference(q, k, v, causal=causal)
    assert torch.allclose(out.cpu().float(), ref.float(), atol=1e-2, rtol=1e-2)
    r = orc.check(out.cpu(), orc.attention_fp32(q, k, v, causal=causal)[0])
    assert r["ok"], r


def test_python_api_gqa_and_lse(sm100):
    q, k, v = _inputs(2, 8, 2, 300, 128, True)
    o, lse = fa.flash_attention_forward(q.cuda(), k.cuda(), v.cuda(), causal=True, return_lse=True)
    ref_o, ref_l = orc.attention_fp32(q, k, v, causal=True)
    assert orc.check(o.cpu(), ref_o)["ok"]
    assert orc.check_lse(lse.cpu(), ref_l)["ok"]
    assert lse.dtype == torch.float32 and lse.shape == (2, 8, 300)


def test_python_api_default_scale_bf16_and_noncontiguous(sm100):
    q, k, v = _inputs(1, 4, 4, 257, 64, False, dtype=torch.bfloat16)
    qd = q.cuda().transpose(1, 2).contiguous().transpose(1, 2)  # non-contiguous view
    assert not qd.is_contiguous()
    o = fa.flash_attention_forward(qd, k.cuda(), v.cuda())
    ref_o, _ = orc.attention_fp32(q, k, v, causal=False, scale=1 / 8.0)
    assert orc.check(o.cpu(), ref_o, atol=1.6e-2, rtol=2e-2)["ok"]
    assert o.dtype == torch.bfloat16


def test_backward_blocked(sm100):
    q, k, v = (t.cuda() for t in _inputs(1, 8, 8, 128, 64))
    q.requires_grad_(True)
    out = fa.flash_attention_forward(q, k, v)
    with pytest.raises(NotImplementedError, match="Backward pass is not implemented"):
        out.sum().backward()


def test_ablation_exports_route_to_kernel(sm100):
    q, k, v = (t.cuda() for t in _inputs(1, 4, 4, 256, 64, True))
    base = C.flash_attention_forward(q, k, v, True, 0.125)
    assert torch.equal(C.flash_attention_forward_scalar(q, k, v, True, 0.125), base)
    assert torch.equal(C.flash_attention_forward_wmma_qk(q, k, v, True, 0.125), base)
    q128 = torch.zeros(1, 1, 16, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim=64 only"):
        C.flash_attention_forward_scalar(q128, q128, q128, False, 1.0)
    with pytest.raises(RuntimeError, match="must be FP16"):
        C.flash_attention_forward_scalar(q.float(), k, v, False, 1.0)


@pytest.mark.parametrize("N,causal", [(1, True), (17, False), (128, True), (300, False)])
def test_naive_attention(sm100, N, causal):
    """Materialised attention (reference naive_attention.cu) against the oracle."""
    q, k, v = _inputs(2, 3, 3, N, 64, causal, seed=N)
    out = C.naive_attention_forward(q.cuda(), k.cuda(), v.cuda(), causal, 0.125)
    ref, _ = orc.attention_fp32(q, k, v, causal=causal, scale=0.125)
    assert orc.check(out.cpu(), ref)["ok"]
    with pytest.raises(RuntimeError, match="identical shapes"):
        C.naive_attention_forward(q.cuda(), k[:, :1].cuda(), v[:, :1].cuda(), causal, 0.125)


def test_llama_patch_on_gpu(sm100):
    from flash_attention_sm75 import llama_attention_replacement as patch
    q, k, v = (t.cuda() for t in _inputs(1, 8, 2, 64, 64, True))
    qd = q[:, :, -3:].contiguous()  # 3 new queries against 64 cached keys
    patch.reset_stats()
    patch.apply_patch()
    try:
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        dec = F.scaled_dot_product_attention(qd[:, :, :1], k, v, enable_gqa=True)  # decode
        chk = F.scaled_dot_product_attention(qd, k, v, is_causal=True, enable_gqa=True)
    finally:
        patch.remove_patch()
    ref, _ = orc.attention_fp32(q.cpu(), k.cpu(), v.cpu(), causal=True)
    assert orc.check(out.cpu(), ref)["ok"]
    s = patch.patch_stats()
    assert s["flash"] == 3 and s["flash_kvcache"] == 2 and s["fallback"] == 0
    # decode: all keys; chunk with is_causal: SDPA's top-left rule (key j <= query i)
    ref_d, _ = orc.attention_fp32(qd[:, :, :1].cpu(), k.cpu(), v.cpu())
    assert orc.check(dec.cpu(), ref_d)["ok"]
    ref_c, _ = orc.attention_fp32(qd.cpu(), k.cpu(), v.cpu(), causal=True, causal_offset=0)
    assert orc.check(chk.cpu(), ref_c)["ok"]
    assert torch.allclose(chk.float(), patch._original_sdpa(qd, k, v, is_causal=True,
                                                            enable_gqa=True).float(),
                          atol=1e-2, rtol=1e-2)
    # reference behaviour on request: decode goes to SDPA
    patch.reset_stats()
    patch.apply_patch(kvcache=False)
    try:
        F.scaled_dot_product_attention(qd[:, :, :1], k, v, enable_gqa=True)
    finally:
        patch.remove_patch()
    assert patch.patch_stats()["fallback_reasons"] == {"kvcache_decode": 1}


def test_current_stream_semantics(sm100):
    q, k, v = (t.cuda() for t in _inputs(2, 8, 8, 2048, 128))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        o1 = C.flash_attention_forward(q, k, v, False, 0.088)
    s.synchronize()
    o2 = C.flash_attention_forward(q, k, v, False, 0.088)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert C.device_status(False) == 0


@pytest.mark.parametrize("B,Hq,Hkv,N,d,causal,chunks", [
    (2, 8, 2, 300, 128, True, 16), (1, 4, 4, 1024, 64, False, 3), (3, 6, 3, 200, 64, True, 1)])
def test_host_pipeline_matches_device_path(sm100, B, Hq, Hkv, N, d, causal, chunks):
    """Host buffers in and out, copies overlapped per (batch, KV-head group)
    chunk: the same kernel per head, so bit-identical to the device call."""
    q, k, v = _inputs(B, Hq, Hkv, N, d, causal)
    ref = fa.flash_attention_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal).cpu()
    out = fa.flash_attention_forward_host(q.pin_memory(), k.pin_memory(), v.pin_memory(),
                                          causal=causal, chunks=chunks)
    assert not out.is_cuda and torch.equal(out, ref)
    pre = torch.zeros_like(q).pin_memory()
    out2 = fa.flash_attention_forward_host(q, k, v, causal=causal, out=pre)  # pageable inputs
    assert out2 is pre and torch.equal(pre, ref)


@pytest.mark.parametrize("causal", [False, True])
def test_host_pipeline_large_matches_oracle(sm100, causal):
    """A size whose halving slices (16, 8, 4, 2, 1, 1 KV-head groups, spanning
    batch entries) run other kernels than the single device call (persistent
    pair kernel for the large slices, tile kernel for the small ones): every
    batch entry and a head of every slice checked against the oracle on
    sampled rows, within the parity tolerance."""
    B, Hq, Hkv, N, d = 4, 32, 8, 2048, 128
    q, k, v = _inputs(B, Hq, Hkv, N, d, causal)
    out = fa.flash_attention_forward_host(q.pin_memory(), k.pin_memory(), v.pin_memory(),
                                          causal=causal)
    assert not out.is_cuda and torch.isfinite(out).all()
    rows = orc.sample_rows(N, 40, seed=4)
    # heads 0, 31 of each batch entry plus the first head of the slices that
    # start inside the batch (units 16, 24, 28, 30, 31 -> b = 2, 3, 3, 3, 3)
    checks = {(b, h) for b in range(B) for h in (0, Hq - 1)}
    checks |= {(u // Hkv, (u % Hkv) * (Hq // Hkv)) for u in (16, 24, 28, 30, 31)}
    for b, h in sorted(checks):
        hk = h // (Hq // Hkv)
        ref_o, _ = orc.attention_fp32(q[b:b + 1, h:h + 1], k[b:b + 1, hk:hk + 1],
                                      v[b:b + 1, hk:hk + 1], causal=causal, rows=rows)
        r = orc.check(out[b:b + 1, h:h + 1, rows], ref_o)
        assert r["ok"], (b, h, r)
