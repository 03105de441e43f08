"""Stage tests of the forward kernel's building blocks (lib/libfa_selftest.so,
built from csrc/fa_selftest.cu with the kernel's own device code):

* the FMA-pipe polynomial exp2 against CUDA's exp2f over a dense sweep of
  its domain, plus inputs below it (clamped, never NaN);
* the register softmax stage of one 128-key tile per row — the known-answer
  test the reference runs on its warp softmax
  (flash-attention-sm75-fused/src/test_warp_softmax.cu:144-241: uniform
  scores in [-2, 2), scales 1/sqrt(16), 1 and 1/sqrt(64)) — here with the
  kernel's MUFU / polynomial split, the diagonal-tile mask and f16/bf16
  packing;
* single-tile tcgen05 products through TMA and the kernel's descriptors
  (S = Q.K^T from shared memory, O = P.V with P in tensor memory), against
  torch.matmul in fp32 — the layout checks of the reference's probes
  (probe_layout.cu).
"""
import ctypes
import math
import os

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SELFTEST = os.path.join(REPO, "flash-attention-sm75-register-fused_b200", "lib",
                        "libfa_selftest.so")

pytestmark = pytest.mark.gpu

_vp, _int, _float = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def _lib():
    lib = ctypes.CDLL(SELFTEST)
    lib.fa_selftest_exp2.argtypes = [_vp, _vp, _vp, _vp, _int, _vp]
    lib.fa_selftest_softmax.argtypes = [_vp, _vp, _int, _float, _int, _vp, _vp, _vp, _vp, _vp]
    lib.fa_selftest_mma.argtypes = [_vp, _vp, _vp, _int, _int, _int, _vp]
    for f in (lib.fa_selftest_exp2, lib.fa_selftest_softmax, lib.fa_selftest_mma):
        f.restype = _int
    return lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_exp2_polynomial_matches_exp2f(sm100):
    lib = _lib()
    t = torch.linspace(-126.0, 64.0, 1 << 21, dtype=torch.float32)
    g = torch.Generator().manual_seed(3)
    t = torch.cat([t, torch.rand(1 << 16, generator=g) * 190.0 - 126.0,
                   torch.tensor([0.0, -0.5, 0.5, -126.0, 64.0, 1e-7, -1e-7, 0.49999997])])
    if t.numel() % 2:
        t = torch.cat([t, torch.zeros(1)])
    td = t.cuda()
    yp, ym, yr = torch.empty_like(td), torch.empty_like(td), torch.empty_like(td)
    assert lib.fa_selftest_exp2(_p(td), _p(yp), _p(ym), _p(yr), td.numel(), _stream()) == 0
    yp, ym, yr = yp.cpu().double(), ym.cpu().double(), yr.cpu().double()
    assert torch.isfinite(yp).all() and (yp > 0).all()
    # Relative error <= 1e-4 (7.5e-5 polynomial error, fp32 evaluation) wherever
    # the result is a normal number.  Within 1e-3 of t = -126 the polynomial's
    # value below 1.0 lands in the subnormal range, where adding n to the
    # exponent field drops the implicit leading bit (1.4e-4 relative at
    # t = -126); such P values round to 0 in f16/bf16 anyway, so that binade
    # is held to an absolute bound.
    normal = t.double() > -125.999
    rel = ((yp - yr).abs() / yr)[normal].max().item()
    assert rel <= 1e-4, rel
    assert ((yp - yr).abs()[~normal] <= 2e-4 * 2.0 ** -126).all()
    rel_mufu = ((ym - yr).abs() / yr).max().item()
    assert rel_mufu <= 1e-6, rel_mufu
    # exact powers of two: the polynomial's value at f = 0 times 2^n
    ints = torch.arange(-125, 65, dtype=torch.float32)
    di = ints.cuda()
    a, b, c = torch.empty_like(di), torch.empty_like(di), torch.empty_like(di)
    assert lib.fa_selftest_exp2(_p(di), _p(a), _p(b), _p(c), di.numel(), _stream()) == 0
    assert (((a.cpu().double() - c.cpu().double()).abs() / c.cpu().double()) <= 1e-4).all()


def test_exp2_polynomial_below_its_domain_stays_finite(sm100):
    """Scores far below the running max (masked keys are -inf only on the
    MUFU path, but large negative exponents reach the polynomial): the input
    is clamped at -126, so the result is a tiny non-negative number, never a
    NaN or a wrapped exponent."""
    lib = _lib()
    t = torch.tensor([-126.5, -127.0, -140.0, -1e4, -3e38, float("-inf"), -126.0, -125.9],
                     dtype=torch.float32).cuda()
    yp, ym, yr = torch.empty_like(t), torch.empty_like(t), torch.empty_like(t)
    assert lib.fa_selftest_exp2(_p(t), _p(yp), _p(ym), _p(yr), t.numel(), _stream()) == 0
    yp = yp.cpu()
    assert torch.isfinite(yp).all()
    assert (yp >= 0).all() and (yp <= 2.0 ** -125).all()


def _softmax_ref(s, lim, sl):
    """The tile stage in float64 from the fp32 inputs: unmasked rows m =
    fp32(max(s)) * sl; masked rows m = max over kept keys of fp32(s * sl);
    p = 2^(s*sl - m) (0 past lim), sum over the row."""
    s32 = s.astype(np.float32)
    sl32 = np.float32(sl)
    rows = s.shape[0]
    m = np.empty(rows, np.float32)
    p = np.zeros_like(s, dtype=np.float64)
    for r in range(rows):
        L = int(lim[r])
        if L >= 128:
            m[r] = np.float32(s32[r].max()) * sl32
            p[r] = np.exp2(s32[r].astype(np.float64) * float(sl32) - float(m[r]))
        else:
            x = (s32[r] * sl32).astype(np.float32)
            m[r] = x[:L].max()
            p[r, :L] = np.exp2(x[:L].astype(np.float64) - float(m[r]))
    return m, p, p.sum(1)


@pytest.mark.parametrize("bf16", [False, True])
def test_softmax_stage_known_answer(sm100, bf16):
    lib = _lib()
    rng = np.random.default_rng(1234)
    blocks, lims, sls = [], [], []
    # the reference KAT's inputs and scales (uniform in [-2, 2)), unmasked
    for scale in (1.0 / math.sqrt(16.0), 1.0, 1.0 / math.sqrt(64.0)):
        blocks.append((rng.random((128, 128)) - 0.5) * 4.0)
        lims.append(np.full(128, 128))
        sls.append(scale * 1.4426950408889634)
    # attention-sized scores with outliers, and masked (diagonal-tile) rows
    x = rng.standard_normal((128, 128)) * 11.3
    x[::7, 5] += 60.0
    blocks.append(x)
    lims.append(np.full(128, 128))
    sls.append(1.4426950408889634 / math.sqrt(128.0))
    blocks.append(rng.standard_normal((128, 128)) * 8.0)
    lims.append(np.arange(1, 129))  # row r keeps keys < r + 1
    sls.append(1.4426950408889634 / math.sqrt(64.0))
    for s_np, lim_np, sl in zip(blocks, lims, sls):
        s = torch.tensor(s_np, dtype=torch.float32).cuda()
        lim = torch.tensor(lim_np, dtype=torch.int32).cuda()
        m = torch.empty(128, device="cuda")
        p = torch.empty(128, 128, device="cuda")
        p16 = torch.empty(128, 64, dtype=torch.int32, device="cuda")
        ssum = torch.empty(128, device="cuda")
        assert lib.fa_selftest_softmax(_p(s), _p(lim), 128, sl, int(bf16), _p(m), _p(p), _p(p16),
                                       _p(ssum), _stream()) == 0
        m_ref, p_ref, sum_ref = _softmax_ref(s_np, lim_np, sl)
        assert np.array_equal(m.cpu().numpy(), m_ref)               # same fp32 max, bit-exact
        pg = p.cpu().double().numpy()
        assert np.all(np.abs(pg - p_ref) <= 1e-4 * p_ref + 1e-30)  # MUFU / polynomial exp2
        assert np.all(pg[p_ref == 0] == 0)                         # masked keys
        assert np.allclose(ssum.cpu().double().numpy(), pg.sum(1), rtol=1e-5, atol=0)
        assert np.allclose(sum_ref, pg.sum(1), rtol=1e-4, atol=0)
        # packing: round-to-nearest of the fp32 P into f16 / bf16 pairs
        dt = torch.bfloat16 if bf16 else torch.float16
        packed = p.cpu().to(dt).view(torch.int16).view(128, 64, 2)
        got = p16.cpu().view(torch.int16).view(128, 64, 2)
        assert torch.equal(got, packed)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bf16", [False, True])
def test_tcgen05_tile_qk_from_shared_memory(sm100, d, bf16):
    """S = A.B^T, 128 x 128 x d, both operands TMA-loaded with the kernel's
    128-byte-swizzled K-major layout and descriptors."""
    lib = _lib()
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(d + 7 * bf16)
    a = torch.randn(128, d, generator=g).to(dt)
    b = torch.randn(128, d, generator=g).to(dt)
    out = torch.empty(128, 128, device="cuda")
    assert lib.fa_selftest_mma(_p(a.cuda()), _p(b.cuda()), _p(out), 0, d, int(bf16),
                               _stream()) == 0
    ref = a.double() @ b.double().T
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= 1e-3 * max(1.0, ref.abs().max().item()), err


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("bf16", [False, True])
def test_tcgen05_tile_pv_from_tensor_memory(sm100, d, bf16):
    """O = P.V, 128 x d x 128 keys, P stored to tensor memory as packed
    pairs (the softmax's layout) and V read MN-major from shared memory."""
    lib = _lib()
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(d + 11 * bf16)
    p = torch.rand(128, 128, generator=g).to(dt)
    v = torch.randn(128, d, generator=g).to(dt)
    pd, vd = p.cuda(), v.cuda()
    out = torch.empty(128, d, device="cuda")
    assert lib.fa_selftest_mma(_p(pd), _p(vd), _p(out), 1, d, int(bf16), _stream()) == 0
    ref = p.double() @ v.double()
    err = (out.cpu().double() - ref).abs().max().item()
    assert err <= 1e-3 * max(1.0, ref.abs().max().item()), err
    # a key's contribution lands in the right column block: one-hot P picks V rows
    onehot = torch.zeros(128, 128)
    onehot[torch.arange(128), torch.arange(128).flip(0)] = 1.0
    assert lib.fa_selftest_mma(_p(onehot.to(dt).cuda()), _p(vd), _p(out), 1, d, int(bf16),
                               _stream()) == 0
    assert torch.equal(out.cpu(), v.float().flip(0))
