"""Parity of fa_fwd_varlen (packed cu_seqlens batches) and fa_fwd_padded
(padded batches with per-entry row ranges) with the CPU oracle, through the
C ABI, plus the Python API and bitwise identities with fa_fwd.

Tolerance: as the forward tests, |err| <= 2e-3 + 1e-2 |ref| for fp16 O (bf16:
1.6e-2 + 2e-2 |ref|) against the fp32 oracle, LSE within 1e-4 absolute.
"""
import pytest
import torch

import flash_attention_sm75 as fa
from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu


def _check_o(got, ref, dtype=torch.float16):
    a, r = (1.6e-2, 2e-2) if dtype == torch.bfloat16 else (2e-3, 1e-2)
    err = (got.float().cpu() - ref).abs()
    assert torch.isfinite(got.float()).all()
    assert (err <= a + r * ref.abs()).all(), err.max().item()


def _check_lse(got, ref):
    got = got.cpu()
    fin = torch.isfinite(ref)
    assert torch.equal(torch.isfinite(got), fin)
    assert (got[~fin] == ref[~fin]).all()
    if fin.any():
        assert (got[fin] - ref[fin]).abs().max().item() <= 1e-4


def _packed(Hq, Hkv, d, lq, lk, seed, dtype=torch.float16):
    """Packed Q [sum(lq), Hq, d], K/V [sum(lk), Hkv, d] and the offsets."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(lq), Hq, d, generator=g).to(dtype)
    k = torch.randn(sum(lk), Hkv, d, generator=g).to(dtype)
    v = torch.randn(sum(lk), Hkv, d, generator=g).to(dtype)
    cu_q, cu_k = [0], [0]
    for a, b in zip(lq, lk):
        cu_q.append(cu_q[-1] + a)
        cu_k.append(cu_k[-1] + b)
    return q, k, v, cu_q, cu_k


VARLEN_CASES = [
    # Hq, Hkv, d, query lengths, key lengths
    (2, 2, 64, [5, 130, 1], [5, 130, 1]),
    (4, 1, 128, [17, 0, 64], [40, 3, 64]),
    (4, 2, 64, [1, 1, 1, 1], [100, 7, 256, 1]),
    (2, 1, 64, [50, 20], [10, 20]),
    (8, 2, 128, [300, 513, 1, 256, 77], [300, 513, 1, 256, 77]),
    (2, 2, 64, [129, 40], [0, 40]),
]


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", VARLEN_CASES, ids=[str(c) for c in VARLEN_CASES])
def test_varlen_matches_oracle(sm100, case, mode):
    Hq, Hkv, d, lq, lk = case
    q, k, v, cu_q, cu_k = _packed(Hq, Hkv, d, lq, lk, seed=sum(lq) + 3 * mode)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    o = torch.full_like(qc, float("nan"))
    lse = torch.full((Hq, q.size(0)), float("nan"), device="cuda")
    cq = torch.tensor(cu_q, dtype=torch.int32, device="cuda")
    ck = torch.tensor(cu_k, dtype=torch.int32, device="cuda")
    rc = abi.fa_fwd_varlen(qc, kc, vc, o, lse, cq, ck, max(lq), max(lk), causal=mode)
    assert rc == 0, abi.load().fa_error_string(rc)
    torch.cuda.synchronize()
    assert abi.load().fa_device_status(1) == 0
    ro, rl = orc.attention_varlen_fp32(q, k, v, cu_q, cu_k, causal_mode=mode)
    _check_o(o, ro)
    _check_lse(lse, rl)


def test_varlen_bf16_and_python_api(sm100):
    q, k, v, cu_q, cu_k = _packed(4, 2, 128, [200, 31, 400], [200, 31, 400], seed=1,
                                  dtype=torch.bfloat16)
    o, lse = fa.flash_attention_varlen_forward(q.cuda(), k.cuda(), v.cuda(), cu_q, cu_k, 400, 400,
                                               causal=True, return_lse=True)
    ro, rl = orc.attention_varlen_fp32(q, k, v, cu_q, cu_k, causal_mode=1)
    _check_o(o, ro, torch.bfloat16)
    _check_lse(lse, rl)


def test_varlen_one_sequence_is_fa_fwd(sm100):
    """One sequence through the packed layout gives fa_fwd's bits."""
    Hq, Hkv, N, d = 8, 2, 700, 128
    q, k, v, cu_q, cu_k = _packed(Hq, Hkv, d, [N], [N], seed=5)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    for causal in (False, True):
        o = fa.flash_attention_varlen_forward(qc, kc, vc, cu_q, cu_k, N, N, causal=causal)
        o4 = torch.empty(1, Hq, N, d, dtype=q.dtype, device="cuda")
        lse4 = torch.empty(1, Hq, N, device="cuda")
        assert abi.fa_fwd(qc.permute(1, 0, 2)[None].contiguous(),
                          kc.permute(1, 0, 2)[None].contiguous(),
                          vc.permute(1, 0, 2)[None].contiguous(), o4, lse4, causal=causal) == 0
        assert torch.equal(o, o4[0].permute(1, 0, 2))


def test_varlen_large_random(sm100):
    g = torch.Generator().manual_seed(9)
    lens = [int(x) for x in torch.randint(1, 2049, (6,), generator=g)] + [2048, 1]
    q, k, v, cu_q, cu_k = _packed(8, 8, 128, lens, lens, seed=2)
    o = fa.flash_attention_varlen_forward(q.cuda(), k.cuda(), v.cuda(), cu_q, cu_k, max(lens),
                                          max(lens), causal=True)
    ro, _ = orc.attention_varlen_fp32(q, k, v, cu_q, cu_k, causal_mode=1)
    _check_o(o, ro)


PADDED_CASES = [
    # B, Hq, Hkv, Nq, Nk, d, q ranges, k ranges
    (3, 2, 2, 100, 100, 64, [(0, 100), (30, 100), (0, 57)], [(0, 100), (30, 100), (0, 57)]),
    (2, 4, 1, 1, 300, 128, [(0, 1), (0, 1)], [(44, 300), (0, 129)]),
    (2, 4, 2, 130, 260, 64, [(0, 130), (5, 130)], [(10, 250), (0, 260)]),
    (2, 8, 2, 600, 600, 128, [(0, 600), (333, 600)], [(0, 600), (333, 600)]),
    (2, 2, 1, 64, 64, 64, [(0, 64), (10, 10)], [(0, 64), (0, 0)]),
]


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", PADDED_CASES, ids=[str(c[:6]) for c in PADDED_CASES])
def test_padded_matches_oracle(sm100, case, mode):
    B, Hq, Hkv, Nq, Nk, d, qr, kr = case
    g = torch.Generator().manual_seed(Nq + Nk + mode)
    q = torch.randn(B, Hq, Nq, d, generator=g).half()
    k = torch.randn(B, Hkv, Nk, d, generator=g).half()
    v = torch.randn(B, Hkv, Nk, d, generator=g).half()
    rng = [torch.tensor(x, dtype=torch.int32, device="cuda") for x in
           ([a for a, _ in qr], [b for _, b in qr], [a for a, _ in kr], [b for _, b in kr])]
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    o = torch.full_like(qc, float("nan"))
    lse = torch.full((B, Hq, Nq), float("nan"), device="cuda")
    rc = abi.fa_fwd_padded(qc, kc, vc, o, lse, *rng, causal=mode)
    assert rc == 0, abi.load().fa_error_string(rc)
    torch.cuda.synchronize()
    ro, rl = orc.attention_padded_fp32(q, k, v, *[r.cpu() for r in rng], causal_mode=mode)
    inside = torch.zeros(B, Hq, Nq, dtype=torch.bool)
    for b, (a, e) in enumerate(qr):
        inside[b, :, a:e] = True
    # rows outside the query ranges are not written by the C ABI
    assert torch.isnan(o.float().cpu()[~inside]).all() and torch.isnan(lse.cpu()[~inside]).all()
    _check_o(o.cpu()[inside], ro[inside])
    _check_lse(lse.cpu()[inside], rl[inside])
    # the Python API returns O = 0 / LSE = -inf there
    po, pl = fa.flash_attention_forward_padded(qc, kc, vc, *rng, causal=mode != 0,
                                               causal_alignment="top_left" if mode == 2
                                               else "bottom_right", return_lse=True)
    assert torch.equal(po[inside], o[inside])
    assert (po.cpu()[~inside] == 0).all() and torch.isinf(pl.cpu()[~inside]).all()


def test_padded_full_ranges_is_fa_fwd(sm100):
    """Full ranges give fa_fwd's bits when both run the same kernel on the same
    tiles: the tile kernel, which the padded path takes at this size and
    FA_DEBUG_TILE_KERNEL gives fa_fwd (whose own non-causal d=64 default here
    is dual-tile items)."""
    B, Hq, Hkv, N, d = 2, 8, 4, 1000, 64
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(B, h, N, d, generator=g).half().cuda() for h in (Hq, Hkv, Hkv))
    lib = abi.load()
    for causal in (False, True):
        o = fa.flash_attention_forward_padded(q, k, v, [0, 0], [N, N], [0, 0], [N, N],
                                              causal=causal)
        o2 = torch.empty_like(q)
        lib.fa_set_debug_flags(8)  # FA_DEBUG_TILE_KERNEL
        try:
            assert abi.fa_fwd(q, k, v, o2, None, causal=causal) == 0
        finally:
            lib.fa_set_debug_flags(0)
        assert torch.equal(o, o2)


def test_ranges_are_clamped(sm100):
    """Offsets outside the tensors are clamped, never followed."""
    q, k, v, _, _ = _packed(2, 2, 64, [64], [64], seed=3)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    o = torch.zeros_like(qc)
    cq = torch.tensor([-5, 1000], dtype=torch.int32, device="cuda")
    ck = torch.tensor([0, 1000], dtype=torch.int32, device="cuda")
    assert abi.fa_fwd_varlen(qc, kc, vc, o, None, cq, ck, 64, 64) == 0
    torch.cuda.synchronize()
    ro, _ = orc.attention_varlen_fp32(q, k, v, [0, 64], [0, 64])
    _check_o(o, ro)


def test_patch_routes_padding_masks(sm100):
    """The SDPA patch sends a padded batch's mask (bool or additive) to the
    padded kernel and matches SDPA on every row; other masks fall back."""
    import torch.nn.functional as F
    from flash_attention_sm75 import llama_attention_replacement as patch
    from tests.test_varlen_cpu import padded_mask
    B, Hq, Hkv, N, d = 3, 8, 2, 300, 128
    g = torch.Generator().manual_seed(8)
    q = torch.randn(B, Hq, N, d, generator=g).half().cuda()
    k = torch.randn(B, Hkv, N, d, generator=g).half().cuda()
    v = torch.randn(B, Hkv, N, d, generator=g).half().cuda()
    rng = [(0, N), (120, N), (0, 77)]
    m = padded_mask(B, N, N, rng, rng, 1).cuda()
    ref = patch._original_sdpa(q, k, v, attn_mask=m, enable_gqa=True).float()
    patch.reset_stats()
    patch.apply_patch()
    try:
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=m, enable_gqa=True)
        add = torch.zeros(m.shape, dtype=torch.float16, device="cuda").masked_fill(
            ~m, torch.finfo(torch.float16).min)
        out_add = F.scaled_dot_product_attention(q, k, v, attn_mask=add, enable_gqa=True)
        hole = m.clone()
        hole[0, 0, 200, 3] = False
        F.scaled_dot_product_attention(q, k, v, attn_mask=hole, enable_gqa=True)
        s = patch.patch_stats()
    finally:
        patch.remove_patch()
    assert s["flash_masked"] == 2 and s["fallback_reasons"] == {"has_attn_mask": 1}
    # rows that see a key match SDPA; fully masked (padding) rows are zeros
    # here, while SDPA's CUDA kernels leave implementation-defined values there
    seen = m[:, 0].any(-1)[:, None, :, None].expand_as(ref)
    for o in (out, out_add):
        err = (o.float() - ref).abs()
        assert (err <= 2e-3 + 1e-2 * ref.abs())[seen].all(), err[seen].max().item()
        assert (o[~seen] == 0).all()
