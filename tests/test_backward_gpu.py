"""Parity of the sm_100a backward (fa_bwd through the C ABI, and the
flash_attention autograd path) with the CPU oracle's fp32 gradients.

Tolerance: dQ, dK, dV are rounded to fp16 once and are computed from P and dS
rounded to fp16 (as in every FlashAttention backward), so each element must
satisfy |err| <= 1e-4 + 1e-2 * max|ref| + 2e-2 * |ref| against the fp32
oracle (bf16: 2.5e-2 and 5e-2); the 1e-4 floor covers gradients that are
exactly 0 in fp32 (N = 1: dS = dP - D = 0) and come out as rounding residue.
"""
import math

import pytest
import torch

import flash_attention_sm75 as fa
from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu


def _inputs(B, Hq, Hkv, N, d, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, N, d, generator=g).to(dtype)
    k = torch.randn(B, Hkv, N, d, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, d, generator=g).to(dtype)
    do = torch.randn(B, Hq, N, d, generator=g).to(dtype)
    return q, k, v, do


def _check(got, ref, dtype):
    a, r = (2.5e-2, 5e-2) if dtype == torch.bfloat16 else (1e-2, 2e-2)
    err = (got.float().cpu() - ref).abs()
    bound = 1e-4 + a * ref.abs().max() + r * ref.abs()
    assert torch.isfinite(got.float()).all()
    assert (err <= bound).all(), (err.max().item(), ref.abs().max().item())


def _run_bwd(q, k, v, do, causal):
    qc, kc, vc, doc = (t.cuda() for t in (q, k, v, do))
    o = torch.empty_like(qc)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device="cuda")
    assert abi.fa_fwd(qc, kc, vc, o, lse, causal=causal) == 0
    dq, dk, dv = torch.empty_like(qc), torch.empty_like(kc), torch.empty_like(vc)
    rc = abi.fa_bwd(qc, kc, vc, o, doc, lse, dq, dk, dv, causal=causal)
    assert rc == 0, abi.load().fa_error_string(rc)
    torch.cuda.synchronize()
    assert abi.load().fa_device_status(1) == 0
    return dq, dk, dv


CASES = [
    # B, Hq, Hkv, N, d, causal
    (1, 2, 2, 128, 64, False), (1, 2, 2, 128, 128, True), (1, 1, 1, 1, 64, False),
    (1, 2, 2, 17, 128, True), (2, 4, 2, 200, 64, True), (1, 4, 1, 300, 128, False),
    (2, 2, 2, 384, 64, False), (1, 8, 2, 256, 128, True), (1, 3, 3, 513, 64, True),
    # causal launch order groups 4 heads: 9 KV heads / 18 query heads leave a partial last group
    (3, 6, 3, 600, 64, True),
]


@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_backward_matches_oracle(sm100, case):
    B, Hq, Hkv, N, d, causal = case
    q, k, v, do = _inputs(B, Hq, Hkv, N, d, seed=sum(case))
    dq, dk, dv = _run_bwd(q, k, v, do, causal)
    rq, rk, rv = orc.attention_grads_fp32(q, k, v, do, causal=causal)
    _check(dq, rq, torch.float16)
    _check(dk, rk, torch.float16)
    _check(dv, rv, torch.float16)


def test_backward_bf16(sm100):
    q, k, v, do = _inputs(1, 4, 2, 200, 128, seed=3, dtype=torch.bfloat16)
    dq, dk, dv = _run_bwd(q, k, v, do, True)
    rq, rk, rv = orc.attention_grads_fp32(q, k, v, do, causal=True)
    for got, ref in ((dq, rq), (dk, rk), (dv, rv)):
        _check(got, ref, torch.bfloat16)


@pytest.mark.parametrize("d", [64, 128])
def test_backward_large_logits(sm100, d):
    """Scores of several tens (LSE/scale in the hundreds) and a few keys x8, as
    in the C5 inputs: the per-query LSE and D values the dK/dV kernel adds to
    its accumulators keep their precision."""
    q, k, v, do = _inputs(1, 4, 2, 300, d, seed=d)
    q, k = q * 3, k * 3
    k[:, :, ::37] *= 8
    dq, dk, dv = _run_bwd(q, k, v, do, True)
    rq, rk, rv = orc.attention_grads_fp32(q, k, v, do, causal=True)
    for got, ref in ((dq, rq), (dk, rk), (dv, rv)):
        _check(got, ref, torch.float16)


def test_autograd_path(sm100):
    """flash_attention(...).backward() gives the C-ABI gradients; the
    reference-compatible flash_attention_forward still refuses backward."""
    q, k, v, do = _inputs(1, 4, 2, 160, 64, seed=9)
    qg, kg, vg = (t.cuda().requires_grad_(True) for t in (q, k, v))
    out = fa.flash_attention(qg, kg, vg, causal=True)
    out.backward(do.cuda())
    dq, dk, dv = _run_bwd(q, k, v, do, True)
    assert torch.equal(qg.grad, dq) and torch.equal(kg.grad, dk) and torch.equal(vg.grad, dv)
    q2 = q.cuda().requires_grad_(True)
    with pytest.raises(NotImplementedError):
        fa.flash_attention_forward(q2, k.cuda(), v.cuda()).sum().backward()


def test_calls_from_a_fresh_host_thread(sm100):
    """fa_fwd / fa_bwd from a thread that has made no CUDA call yet (as
    PyTorch's autograd worker may be): the library binds the device's primary
    context itself before encoding its tensor maps."""
    import threading
    q, k, v, do = (t.cuda() for t in _inputs(1, 4, 2, 160, 64, seed=5))
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    torch.cuda.synchronize()
    rcs = []

    def work():
        rcs.append(abi.fa_fwd(q, k, v, o, lse, causal=True))
        rcs.append(abi.fa_bwd(q, k, v, o, do, lse, dq, dk, dv, causal=True))

    th = threading.Thread(target=work)
    th.start()
    th.join()
    torch.cuda.synchronize()
    assert rcs == [0, 0], [abi.load().fa_error_string(r) for r in rcs]
    rq, rk, rv = _run_bwd(*(t.cpu() for t in (q, k, v, do)), True)
    assert torch.equal(dq, rq) and torch.equal(dk, rk) and torch.equal(dv, rv)


def test_backward_argument_errors(sm100):
    q, k, v, do = (t.cuda() for t in _inputs(1, 2, 2, 64, 64, seed=1))
    lib = abi.load()
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device="cuda")
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")  # too small
    rc = lib.fa_bwd(abi.ptr(q), abi.ptr(k), abi.ptr(v), abi.ptr(o), abi.ptr(do), abi.ptr(lse),
                    abi.ptr(q), abi.ptr(k), abi.ptr(v), 1, 2, 2, 64, 64, 0.125, 0, 0, abi.ptr(ws),
                    16, abi.stream_ptr())
    assert rc == 1  # FA_ERR_INVALID_ARG: workspace too small
    assert lib.fa_bwd_workspace_bytes(1, 2, 64) == 2 * 2 * 128 * 4 + 2 * 8192


def _padded_grads_ref(q, k, v, do, ranges, causal):
    """fp32 autograd reference of a square padded batch: key j visible to query
    i of entry b iff both lie in the entry's ranges (and j <= i when causal);
    rows without a visible key have output 0."""
    B, Hq, N, d = q.shape
    G = Hq // k.size(1)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    kx, vx = kf.repeat_interleave(G, 1), vf.repeat_interleave(G, 1)
    i = torch.arange(N)[:, None]
    j = torch.arange(N)[None, :]
    mask = torch.zeros(B, 1, N, N, dtype=torch.bool)
    for b, ((q0, q1), (k0, k1)) in enumerate(ranges):
        m = (i >= q0) & (i < q1) & (j >= k0) & (j < k1)
        if causal:
            m &= j <= i
        mask[b, 0] = m
    s = (qf @ kx.transpose(-2, -1)) / math.sqrt(d)
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    (p @ vx).backward(do.float())
    return qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_padded_backward_matches_reference(sm100, d, causal):
    B, Hq, Hkv, N = 3, 4, 2, 200
    q, k, v, do = _inputs(B, Hq, Hkv, N, d, seed=d + causal)
    ranges = [((0, N), (0, N)), ((37, N), (37, N)), ((0, 150), (0, 150))]
    qc, kc, vc, doc = (t.cuda() for t in (q, k, v, do))
    rng = [torch.tensor([r[i][j] for r in ranges], dtype=torch.int32, device="cuda")
           for i in (0, 1) for j in (0, 1)]
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (qc, kc, vc))
    out = fa.flash_attention_padded(qg, kg, vg, *rng, causal=causal)
    out.backward(doc)
    rq, rk, rv = _padded_grads_ref(q, k, v, do, ranges, causal)
    for got, ref in ((qg.grad, rq), (kg.grad, rk), (vg.grad, rv)):
        _check(got, ref, torch.float16)
    # padding: exact zeros
    assert (qg.grad[1, :, :37] == 0).all() and (qg.grad[2, :, 150:] == 0).all()
    assert (kg.grad[1, :, :37] == 0).all() and (vg.grad[2, :, 150:] == 0).all()
    # the C ABI entry point gives the same bits
    o, lse = fa.flash_attention_forward_padded(qc, kc, vc, *rng, causal=causal, return_lse=True)
    dq, dk, dv = torch.empty_like(qc), torch.empty_like(kc), torch.empty_like(vc)
    assert abi.fa_bwd_padded(qc, kc, vc, o, doc, lse, *rng, dq, dk, dv, causal=causal) == 0
    torch.cuda.synchronize()
    assert torch.equal(dq, qg.grad) and torch.equal(dk, kg.grad) and torch.equal(dv, vg.grad)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_varlen_backward_matches_oracle(sm100, d, causal):
    """Packed self-attention batch: gradients of every sequence equal the
    oracle's on that sequence alone."""
    lens = [1, 130, 37, 300, 256]
    Hq, Hkv = 4, 2
    g = torch.Generator().manual_seed(d + 2 * causal)
    T = sum(lens)
    q = torch.randn(T, Hq, d, generator=g).half()
    k = torch.randn(T, Hkv, d, generator=g).half()
    v = torch.randn(T, Hkv, d, generator=g).half()
    do = torch.randn(T, Hq, d, generator=g).half()
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    qg, kg, vg = (t.cuda().requires_grad_(True) for t in (q, k, v))
    out = fa.flash_attention_varlen(qg, kg, vg, cu, max(lens), causal=causal)
    out.backward(do.cuda())
    for i, n in enumerate(lens):
        sl = slice(cu[i], cu[i + 1])
        per = lambda x: x[sl].permute(1, 0, 2)[None]
        rq, rk, rv = orc.attention_grads_fp32(per(q), per(k), per(v), per(do), causal=causal)
        for got, ref in ((qg.grad, rq), (kg.grad, rk), (vg.grad, rv)):
            _check(got[sl].permute(1, 0, 2)[None], ref, torch.float16)
    # the C ABI entry point gives the same bits
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    o, lse = fa.flash_attention_varlen_forward(qc, kc, vc, cu, cu, max(lens), max(lens),
                                               causal=causal, return_lse=True)
    dq, dk, dv = torch.empty_like(qc), torch.empty_like(kc), torch.empty_like(vc)
    cu_t = torch.tensor(cu, dtype=torch.int32, device="cuda")
    assert abi.fa_bwd_varlen(qc, kc, vc, o, do.cuda(), lse, cu_t, max(lens), dq, dk, dv,
                             causal=causal) == 0
    torch.cuda.synchronize()
    assert torch.equal(dq, qg.grad) and torch.equal(dk, kg.grad) and torch.equal(dv, vg.grad)
