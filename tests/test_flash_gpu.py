"""Parity of the sm_100a kernel against the CPU oracle, called through the C ABI.

Tolerance (north star): |O - O_ref| <= 2e-3 + 1e-2*|O_ref| elementwise on
fp16 output against the fp32 oracle (bf16: 1.6e-2 + 2e-2*|ref|, one bf16
rounding), LSE within 1e-4 absolute.  Small shapes are checked in full; the
BASELINE configurations C4/C5 on sampled query rows (oracle row-sampled with
full K/V) plus size-independent properties.
"""
import glob
import math
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu

BF16_ATOL, BF16_RTOL = 1.6e-2, 2e-2


def run(q, k, v, causal, scale=None, want_lse=True):
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device) if want_lse else None
    rc = abi.fa_fwd(q, k, v, o, lse, causal=causal, scale=scale)
    assert rc == 0, abi.load().fa_error_string(rc)
    torch.cuda.synchronize()
    return o, lse


def parity(B, Hq, Hkv, N, d, causal, dtype=torch.float16, seed=0, scale=None, rows=None,
           input_scale=1.0, lse_rtol=0.0):
    cfg = orc.AttnConfig("t", B, Hq, Hkv, N, d, causal, input_scale=input_scale)
    q, k, v = orc.make_inputs(cfg, seed=seed, dtype=dtype)
    o, lse = run(q.cuda(), k.cuda(), v.cuda(), causal, scale)
    ref_o, ref_lse = orc.attention_fp32(q, k, v, causal=causal, scale=scale, rows=rows)
    o, lse = o.cpu(), lse.cpu()
    if rows is not None:
        o, lse = o[:, :, rows], lse[:, :, rows]
    if dtype == torch.bfloat16:
        r = orc.check(o, ref_o, atol=BF16_ATOL, rtol=BF16_RTOL)
    else:
        r = orc.check(o, ref_o)
    rl = orc.check_lse(lse, ref_lse)
    assert r["ok"], r
    if lse_rtol:
        lerr = (lse.float() - ref_lse.float()).abs()
        assert (lerr <= orc.LSE_ATOL + lse_rtol * ref_lse.float().abs()).all(), rl
    else:
        assert rl["ok"], rl
    return r, rl


SMALL = [
    # B, Hq, Hkv, N, d, causal
    (1, 1, 1, 1, 64, False), (1, 1, 1, 1, 128, True), (1, 2, 2, 16, 64, True),
    (1, 2, 2, 17, 128, False), (1, 1, 1, 127, 64, True), (1, 1, 1, 128, 128, True),
    (1, 1, 1, 129, 64, False), (1, 2, 2, 255, 128, True), (1, 1, 1, 256, 64, True),
    (1, 1, 1, 257, 128, False), (2, 3, 3, 384, 64, False), (1, 2, 2, 512, 128, True),
    (1, 1, 1, 1000, 64, True), (2, 2, 2, 1024, 128, False), (1, 8, 8, 1024, 64, True),
    (1, 8, 2, 640, 128, True), (2, 6, 1, 333, 64, False), (1, 4, 4, 2048, 128, True),
    # head counts that are no multiple of the causal launch-order group
    (2, 5, 5, 700, 64, True), (3, 6, 2, 900, 128, True),
]


def test_causal_partial_head_group_many_waves(sm100):
    """A causal launch of more than two waves orders its items pair-major in
    groups of 8 heads: 18 heads x 17 Q pairs = 306 items on 148 SMs leave a
    partial last group of 2 heads, whose rows (and the others') match the
    oracle on sampled rows."""
    c = orc.AttnConfig("t", 1, 18, 6, 4352, 128, True)
    q, k, v = orc.make_inputs(c, seed=17)
    o, lse = run(q.cuda(), k.cuda(), v.cuda(), True)
    o, lse = o.cpu(), lse.cpu()
    rows = orc.sample_rows(c.N, 24, seed=5)
    for h in (0, 7, 8, 15, 16, 17):
        hk = h // 3
        ref_o, ref_l = orc.attention_fp32(q[:, h:h + 1], k[:, hk:hk + 1], v[:, hk:hk + 1],
                                          causal=True, rows=rows)
        assert orc.check(o[:, h:h + 1, rows], ref_o)["ok"], h
        assert orc.check_lse(lse[:, h:h + 1, rows], ref_l)["ok"], h


@pytest.mark.parametrize("B,Hq,Hkv,N,d,causal", SMALL)
def test_parity_small(sm100, B, Hq, Hkv, N, d, causal):
    parity(B, Hq, Hkv, N, d, causal, seed=N + d)


@pytest.mark.parametrize("d,causal", [(64, False), (64, True), (128, False), (128, True)])
def test_parity_bf16(sm100, d, causal):
    parity(2, 4, 2, 700, d, causal, dtype=torch.bfloat16, seed=11)


@pytest.mark.parametrize("scale", [0.0, 0.05, 0.3, -0.125])
def test_parity_custom_scale(sm100, scale):
    parity(1, 2, 2, 300, 64, True, scale=scale, seed=3)


@pytest.mark.parametrize("d,causal,dtype", [(64, False, torch.float16), (128, False, torch.float16),
                                             (128, True, torch.float16),
                                             (128, False, torch.bfloat16)])
def test_parity_wide_score_range(sm100, d, causal, dtype):
    """Scores spanning several hundred log2 units inside unmasked tiles, so that
    exponents far below 2^-126 reach both exponential paths (MUFU and the
    FMA-pipe polynomial) and must come out as zeros, never NaN.  The LSE here
    reaches ~250, where 1e-4 is three fp32 ulps, so LSE gets a relative term
    of 2e-6 (a few ulps of the fp32 score accumulation scaled by 6)."""
    r, _ = parity(1, 2, 2, 512, d, causal, dtype=dtype, scale=6.0, seed=21, lse_rtol=2e-6)
    assert r["finite"]


@pytest.mark.parametrize("name", ["c1", "c2", "c3"])
def test_parity_baseline_configs_full(sm100, name):
    c = orc.CONFIGS[name]
    parity(c.B, c.Hq, c.Hkv, c.N, c.d, c.causal, seed=42, input_scale=c.input_scale)


@pytest.mark.parametrize("name", ["c4", "c5", "c5c"])
def test_parity_baseline_configs_sampled(sm100, name):
    c = orc.CONFIGS[name]
    q, k, v = orc.make_inputs(c, seed=42)
    o, lse = run(q.cuda(), k.cuda(), v.cuda(), c.causal)
    o, lse = o.cpu(), lse.cpu()
    rows = orc.sample_rows(c.N, 96, seed=1)
    # oracle on two (b, h) slices per batch entry to bound CPU time
    for b in range(c.B):
        for h in (0, c.Hq - 1 - b % c.Hq):
            hk = h // (c.Hq // c.Hkv)
            ref_o, ref_l = orc.attention_fp32(q[b:b + 1, h:h + 1], k[b:b + 1, hk:hk + 1],
                                              v[b:b + 1, hk:hk + 1], causal=c.causal, rows=rows)
            r = orc.check(o[b:b + 1, h:h + 1, rows], ref_o)
            rl = orc.check_lse(lse[b:b + 1, h:h + 1, rows], ref_l)
            assert r["ok"], (b, h, r)
            assert rl["ok"], (b, h, rl)
    assert torch.isfinite(o).all()


GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[7:-4] for p in GOLDEN])
def test_golden_through_c_abi(sm100, path):
    z = np.load(path)
    q, k, v = (torch.from_numpy(z[n]) for n in ("q", "k", "v"))
    o, _ = run(q.cuda(), k.cuda(), v.cuda(), bool(z["causal"]), float(z["scale"]))
    ref = torch.from_numpy(z["o_ref"]).float()
    # the reference's own fp16 output: both sides round once to fp16
    err = (o.cpu().float() - ref).abs()
    assert (err <= 3e-3 + 1e-2 * ref.abs()).all(), err.max().item()


def test_full_size_properties(sm100):
    """Size-independent checks at C5's full size: constant V gives O == V
    (to one fp16 rounding: P is rounded before PV, l is summed in fp32), and
    permuting keys (with their values) leaves full attention unchanged."""
    c = orc.CONFIGS["c5"]
    q, k, v = orc.make_inputs(c, seed=42)
    q, k = q.cuda(), k.cuda()
    vc = torch.full_like(k, 0.75)
    o, lse = run(q, k, vc, False)
    assert (o.float() - vc.float()).abs().max().item() <= 4.9e-4
    perm = torch.randperm(c.N, generator=torch.Generator().manual_seed(3)).cuda()
    v = v.cuda()
    o1, l1 = run(q, k, v, False)
    o2, l2 = run(q, k[:, :, perm].contiguous(), v[:, :, perm].contiguous(), False)
    # both are kernel outputs, each within the tolerance of the exact value
    diff = (o1.float() - o2.float()).abs()
    assert (diff <= 2 * (2e-3 + 1e-2 * o1.float().abs())).all(), diff.max().item()
    assert (l1 - l2).abs().max().item() <= 2e-4


def test_causal_row0_is_v0(sm100):
    c = orc.AttnConfig("t", 2, 4, 4, 4096, 128, True)
    q, k, v = orc.make_inputs(c, seed=9)
    o, lse = run(q.cuda(), k.cuda(), v.cuda(), True)
    assert torch.equal(o[:, :, 0].cpu(), v[:, :, 0])
    s0 = (q[:, :, 0].float() * k[:, :, 0].float()).sum(-1) / math.sqrt(128)
    assert (lse[:, :, 0].cpu() - s0).abs().max().item() < 1e-4


def test_deterministic(sm100):
    c = orc.AttnConfig("t", 2, 8, 2, 1500, 128, True)
    q, k, v = (t.cuda() for t in orc.make_inputs(c, seed=4))
    o1, l1 = run(q, k, v, True)
    o2, l2 = run(q, k, v, True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_lse_null_and_stream(sm100):
    c = orc.AttnConfig("t", 1, 4, 4, 384, 64, False)
    q, k, v = (t.cuda() for t in orc.make_inputs(c, seed=1))
    s = torch.cuda.Stream()
    o = torch.empty_like(q)
    with torch.cuda.stream(s):
        rc = abi.fa_fwd(q, k, v, o, None, causal=False, stream=s)
    assert rc == 0
    s.synchronize()
    o2, _ = run(q, k, v, False)
    assert torch.equal(o, o2)
    assert abi.load().fa_device_status(0) == 0


def _spiked_inputs(B, Hq, Hkv, Nq, Nk, d, spikes, dtype=torch.float16, seed=5):
    """Queries in [0.5, 1] and small random keys, except keys at the positions
    `spikes` (ascending), which are constant vectors of growing size: each
    spike lifts a row's running score maximum by ~18 log2 units (above the
    kernel's lazy-rescale threshold of 15), wherever it falls in a K/V tile."""
    g = torch.Generator().manual_seed(seed)
    q = 0.5 + 0.5 * torch.rand(B, Hq, Nq, d, generator=g)
    k = 0.3 * torch.randn(B, Hkv, Nk, d, generator=g)
    v = torch.randn(B, Hkv, Nk, d, generator=g)
    step = 18.0 / (0.75 * math.sqrt(d) * 1.4426950408889634)
    for t, pos in enumerate(spikes):
        k[:, :, pos] = step * (t + 1)
    return q.to(dtype), k.to(dtype), v.to(dtype)


# spike positions (128-key tiles, the first 64 keys of a tile form its early
# part): tile 1 early, tile 2 late, tile 3 early then late, tile 5 last key,
# tile 7 first late key, tile 8 early
SPIKES = [133, 356, 404, 474, 767, 960, 1030]


@pytest.mark.parametrize("d,causal,dtype", [(64, False, torch.float16), (128, False, torch.float16),
                                             (128, True, torch.float16), (64, True, torch.bfloat16)])
def test_parity_late_max_growth(sm100, d, causal, dtype):
    """The running maximum grows by more than the rescale threshold in later
    K/V tiles, in either part of a tile and twice within one: O and l must be
    rescaled consistently whichever part of P was already consumed."""
    q, k, v = _spiked_inputs(1, 4, 2, 1100, 1100, d, SPIKES, dtype)
    o, lse = run(q.cuda(), k.cuda(), v.cuda(), causal)
    ref_o, ref_lse = orc.attention_fp32(q, k, v, causal=causal)
    if dtype == torch.bfloat16:
        r = orc.check(o.cpu(), ref_o, atol=BF16_ATOL, rtol=BF16_RTOL)
    else:
        r = orc.check(o.cpu(), ref_o)
    assert r["ok"], r
    lerr = (lse.cpu() - ref_lse).abs()
    assert (lerr <= orc.LSE_ATOL + 2e-6 * ref_lse.abs()).all(), lerr.max().item()


@pytest.mark.parametrize("Nq,Nk", [(1, 4096), (3, 2500)])
def test_parity_late_max_growth_kvcache(sm100, Nq, Nk):
    """Late max growth in the split-KV (decode) path, where each split and
    each half of a dual split rescales on its own before the combine."""
    spikes = [133, 356, 404, 474, 1279, 2050, 2333]
    q, k, v = _spiked_inputs(2, 8, 2, Nq, Nk, 128, spikes)
    o = torch.empty_like(q).cuda()
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device="cuda")
    rc = abi.fa_fwd_kvcache(q.cuda(), k.cuda(), v.cuda(), o, lse, causal=1, workspace=True)
    assert rc == 0, abi.load().fa_error_string(rc)
    torch.cuda.synchronize()
    ref_o, ref_lse = orc.attention_fp32(q, k, v, causal=True,
                                        causal_offset=orc.kvcache_offset(Nq, Nk, 1))
    r = orc.check(o.cpu(), ref_o)
    assert r["ok"], r
    lerr = (lse.cpu() - ref_lse).abs()
    assert (lerr <= orc.LSE_ATOL + 2e-6 * ref_lse.abs()).all(), lerr.max().item()


# The forward kernels on the same shapes, each forced through its debug flag:
# the pair kernel (two Q tiles per CTA; the default once a launch fills a
# wave), its CTA-pair form (one product for two SMs, d = 128; opt-in) and the
# tile kernel (one Q tile per CTA, S double-buffered; the default for
# launches that would leave SMs idle, except non-causal d=64 ones, which run
# dual-tile items).
FORCED = [(1, 1, 1, 1, 64, True), (1, 2, 2, 17, 128, False), (1, 1, 1, 129, 64, False),
          (1, 2, 2, 255, 128, True), (1, 8, 2, 640, 128, True), (2, 6, 1, 333, 64, False),
          (3, 6, 2, 900, 128, True), (1, 4, 4, 2048, 128, True), (2, 5, 5, 700, 64, True)]


@pytest.mark.parametrize("flag", [2, 8, 8 | 4, 16], ids=["pair", "tile4", "tile2", "pair2"])
@pytest.mark.parametrize("B,Hq,Hkv,N,d,causal", FORCED)
def test_parity_forced_kernel(sm100, flag, B, Hq, Hkv, N, d, causal):
    lib = abi.load()
    lib.fa_set_debug_flags(flag)
    try:
        parity(B, Hq, Hkv, N, d, causal, seed=3 * N + d)
    finally:
        lib.fa_set_debug_flags(0)


@pytest.mark.parametrize("flag", [2, 8, 16], ids=["pair", "tile4", "pair2"])
@pytest.mark.parametrize("d,causal", [(64, True), (128, False), (128, True)])
def test_forced_kernels_bf16_and_outliers(sm100, flag, d, causal):
    """bf16, and K rows x8 (the C5 outliers: late running-max growth and the
    lazy rescale) on a 32-head launch that fills several waves."""
    lib = abi.load()
    lib.fa_set_debug_flags(flag)
    try:
        parity(2, 4, 2, 700, d, causal, dtype=torch.bfloat16, seed=12)
        cfg = orc.AttnConfig("t", 1, 32, 32, 1024, d, causal, k_outlier_frac=0.01)
        q, k, v = orc.make_inputs(cfg, seed=5)
        o, lse = run(q.cuda(), k.cuda(), v.cuda(), causal)
        rows = orc.sample_rows(1024, 64, seed=1)
        ref_o, ref_lse = orc.attention_fp32(q, k, v, causal=causal, rows=rows)
        assert orc.check(o.cpu()[:, :, rows], ref_o)["ok"]
        assert orc.check_lse(lse.cpu()[:, :, rows], ref_lse)["ok"]
    finally:
        lib.fa_set_debug_flags(0)


@pytest.mark.parametrize("d", [64, 128])
def test_wave_tail_items_on_the_tile_kernel(sm100, d):
    """A non-causal launch whose pair-kernel items fill one wave of SMs plus
    a few (80 heads x 2 Q pairs = 160 items on 148 SMs) runs the last items on
    the tile kernel at d=128; at d=64 the launch has no tail split (it runs
    dual-tile items): every head, those included, matches the oracle, and the
    result agrees with the launch without the split (bit for bit at d=64)."""
    lib = abi.load()
    cfg = orc.AttnConfig("t", 1, 80, 80, 512, d, False)
    q, k, v = orc.make_inputs(cfg, seed=21)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o, lse = run(qd, kd, vd, False)
    rows = orc.sample_rows(512, 32, seed=2)
    for h in (0, 71, 72, 79):  # pair items 0, 143, 144 (tail), 159 (tail)
        ref_o, ref_l = orc.attention_fp32(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], rows=rows)
        assert orc.check(o.cpu()[:, h:h + 1, rows], ref_o)["ok"], h
        assert orc.check_lse(lse.cpu()[:, h:h + 1, rows], ref_l)["ok"], h
    lib.fa_set_debug_flags(32)  # FA_DEBUG_NO_TAIL_SPLIT
    try:
        o2, lse2 = run(qd, kd, vd, False)
    finally:
        lib.fa_set_debug_flags(0)
    assert (o.float() - o2.float()).abs().max().item() <= 4e-3
    assert (lse - lse2).abs().max().item() <= 1e-4
    if d == 64:
        assert torch.equal(o, o2) and torch.equal(lse, lse2)


@pytest.mark.parametrize("causal", [False, True])
def test_persistent_pair_kernel_many_rounds(sm100, causal):
    """A launch of >= 16 rounds of pair-kernel items runs persistent CTAs that
    walk several items each (Q buffers refilled across items, barrier phases
    running on; the last two rounds taken from the device-wide counter):
    sampled rows of the first, middle and last heads match the oracle and
    agree bit for bit with one CTA per item and with every round dealt
    statically (an item skipped or dealt twice would show)."""
    lib = abi.load()
    cfg = orc.AttnConfig("t", 2, 600, 600, 512, 64, causal)  # 2400 items = 16.2 rounds
    q, k, v = orc.make_inputs(cfg, seed=31)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o, lse = run(qd, kd, vd, causal)
    rows = orc.sample_rows(512, 24, seed=3)
    for b, h in ((0, 0), (0, 299), (1, 300), (1, 599)):
        ref_o, ref_l = orc.attention_fp32(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                          v[b:b + 1, h:h + 1], causal=causal, rows=rows)
        assert orc.check(o.cpu()[b:b + 1, h:h + 1, rows], ref_o)["ok"], (b, h)
        assert orc.check_lse(lse.cpu()[b:b + 1, h:h + 1, rows], ref_l)["ok"], (b, h)
    for flag in (64, 128):  # FA_DEBUG_NO_PERSIST, FA_DEBUG_STATIC_DEAL
        lib.fa_set_debug_flags(flag)
        try:
            o2, lse2 = run(qd, kd, vd, causal)
        finally:
            lib.fa_set_debug_flags(0)
        assert torch.equal(o, o2), flag
        assert torch.equal(lse, lse2), flag
    assert lib.fa_device_status(0) == 0


@pytest.mark.parametrize("H,N,causal", [(12, 1024, False), (8, 2048, True)])
def test_persistent_two_waves_d64(sm100, H, N, causal):
    """A d=64 launch of between one and two waves of pair items (C2's shape:
    48 heads x 4 Q pairs = 192 items; C3's causal shape: 32 heads x 8 pairs =
    256 items, on 148 SMs) runs persistent CTAs, some of which walk two
    items: every head matches the oracle on sampled rows and the result
    equals one CTA per item bit for bit."""
    lib = abi.load()
    cfg = orc.AttnConfig("t", 4, H, H, N, 64, causal)
    q, k, v = orc.make_inputs(cfg, seed=33)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    lib.fa_set_debug_flags(2)  # FA_DEBUG_PAIR_KERNEL: Q pairs, not dual-tile items
    try:
        o, lse = run(qd, kd, vd, causal)
    finally:
        lib.fa_set_debug_flags(0)
    rows = orc.sample_rows(N, 16, seed=4)
    for b in range(4):
        for h in (0, H // 2 - 1, H - 1):
            ref_o, ref_l = orc.attention_fp32(q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1],
                                              v[b:b + 1, h:h + 1], causal=causal, rows=rows)
            assert orc.check(o.cpu()[b:b + 1, h:h + 1, rows], ref_o)["ok"], (b, h)
            assert orc.check_lse(lse.cpu()[b:b + 1, h:h + 1, rows], ref_l)["ok"], (b, h)
    lib.fa_set_debug_flags(2 | 64)  # FA_DEBUG_PAIR_KERNEL | FA_DEBUG_NO_PERSIST
    try:
        o2, lse2 = run(qd, kd, vd, causal)
    finally:
        lib.fa_set_debug_flags(0)
    assert torch.equal(o, o2)
    assert torch.equal(lse, lse2)
    assert lib.fa_device_status(0) == 0


@pytest.mark.parametrize("B,Hq,Hkv,N,causal,dtype", [
    (1, 2, 2, 256, True, torch.float16),     # two key tiles: tile 0's second group has none
    (2, 3, 3, 1000, False, torch.float16),   # ragged last tile
    (1, 8, 2, 777, True, torch.float16),     # GQA, ragged, causal
    (2, 4, 4, 640, True, torch.bfloat16),
    (4, 12, 12, 1024, False, torch.float16),  # C2's shape: 384 items on 148 CTAs
])
def test_dual_tile_items_d64(sm100, B, Hq, Hkv, N, causal, dtype):
    """d=64 launches as one-Q-tile items whose two softmax groups take halves
    of the keys and merge them inside the CTA (FA_DEBUG_DUAL_TILES; the
    default for C2's shape): O and LSE match the oracle, repeat bit for bit,
    and agree with the launch on Q pairs within the kernel-to-kernel
    tolerance; no watchdog error."""
    lib = abi.load()
    cfg = orc.AttnConfig("t", B, Hq, Hkv, N, 64, causal)
    q, k, v = orc.make_inputs(cfg, seed=N + B, dtype=dtype)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    lib.fa_set_debug_flags(256)  # FA_DEBUG_DUAL_TILES
    try:
        o, lse = run(qd, kd, vd, causal)
        o_again, _ = run(qd, kd, vd, causal)
    finally:
        lib.fa_set_debug_flags(0)
    assert torch.equal(o, o_again)
    rows = None if B * Hq * N <= 8192 else orc.sample_rows(N, 16, seed=6)
    ref_o, ref_l = orc.attention_fp32(q, k, v, causal=causal, rows=rows)
    oc, lc = o.cpu(), lse.cpu()
    if rows is not None:
        oc, lc = oc[:, :, rows], lc[:, :, rows]
    if dtype == torch.bfloat16:
        assert orc.check(oc, ref_o, atol=BF16_ATOL, rtol=BF16_RTOL)["ok"]
    else:
        assert orc.check(oc, ref_o)["ok"]
    assert orc.check_lse(lc, ref_l)["ok"]
    lib.fa_set_debug_flags(2)  # FA_DEBUG_PAIR_KERNEL
    try:
        o2, lse2 = run(qd, kd, vd, causal)
    finally:
        lib.fa_set_debug_flags(0)
    if (B, Hq, N, causal) == (4, 12, 1024, False):
        o3, lse3 = run(qd, kd, vd, causal)  # the default plan: dual-tile items
        assert torch.equal(o, o3) and torch.equal(lse, lse3)
    tol = 2 * (BF16_ATOL if dtype == torch.bfloat16 else 2e-3)
    assert (o.float() - o2.float()).abs().max().item() <= tol
    assert (lse - lse2).abs().max().item() <= 2e-4
    assert lib.fa_device_status(0) == 0
