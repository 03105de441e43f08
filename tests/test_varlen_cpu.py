"""Variable-length (packed, cu_seqlens) and padded-batch attention, CPU side.

The oracle's per-sequence restatements are pinned against PyTorch's own
scaled_dot_product_attention on the CPU in fp32 with explicit boolean masks:
one attention over all packed tokens with a block-diagonal (same sequence)
mask, and a [B, 1, Nq, Nk] padding mask for the padded batch.  Rows that see
no key are NaN in SDPA and O = 0 / LSE = -inf in the oracle; they are checked
separately.  The C entry points' argument errors that need no GPU are checked
through ctypes.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

VARLEN_CASES = [
    # Hq, Hkv, d, query lengths, key lengths
    (2, 2, 64, [5, 130, 1], [5, 130, 1]),
    (4, 1, 128, [17, 0, 64], [40, 3, 64]),
    (4, 2, 64, [1, 1, 1, 1], [100, 7, 256, 1]),
    (2, 1, 64, [50, 20], [10, 20]),
]


def _packed(Hq, Hkv, d, lq, lk, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(lq), Hq, d, generator=g).half()
    k = torch.randn(sum(lk), Hkv, d, generator=g).half()
    v = torch.randn(sum(lk), Hkv, d, generator=g).half()
    cu_q = [0]
    cu_k = [0]
    for a, b in zip(lq, lk):
        cu_q.append(cu_q[-1] + a)
        cu_k.append(cu_k[-1] + b)
    return q, k, v, cu_q, cu_k


def _varlen_mask(cu_q, cu_k, mode):
    Tq, Tk = cu_q[-1], cu_k[-1]
    mask = torch.zeros(Tq, Tk, dtype=torch.bool)
    for b in range(len(cu_q) - 1):
        nq, nk = cu_q[b + 1] - cu_q[b], cu_k[b + 1] - cu_k[b]
        i = torch.arange(nq)[:, None]
        j = torch.arange(nk)[None, :]
        blk = torch.ones(nq, nk, dtype=torch.bool)
        if mode:
            blk = j <= i + orc.kvcache_offset(nq, nk, mode)
        mask[cu_q[b]:cu_q[b + 1], cu_k[b]:cu_k[b + 1]] = blk
    return mask


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", VARLEN_CASES, ids=[str(c) for c in VARLEN_CASES])
def test_varlen_oracle_matches_torch_sdpa(case, mode):
    Hq, Hkv, d, lq, lk = case
    q, k, v, cu_q, cu_k = _packed(Hq, Hkv, d, lq, lk, seed=sum(lq) + mode)
    o, lse = orc.attention_varlen_fp32(q, k, v, cu_q, cu_k, causal_mode=mode)
    mask = _varlen_mask(cu_q, cu_k, mode)
    G = Hq // Hkv
    qh = q.permute(1, 0, 2).float()[None]
    kh = k.permute(1, 0, 2).repeat_interleave(G, dim=0).float()[None]
    vh = v.permute(1, 0, 2).repeat_interleave(G, dim=0).float()[None]
    ref = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask)[0].permute(1, 0, 2)
    seen = mask.any(dim=1)
    assert (o[seen] - ref[seen]).abs().max().item() < 1e-5
    assert (o[~seen] == 0).all() and torch.isinf(lse[:, ~seen]).all()
    S = torch.matmul(qh, kh.transpose(-2, -1))[0] / d ** 0.5
    ref_lse = torch.logsumexp(S.masked_fill(~mask, float("-inf")), dim=-1)
    assert (lse[:, seen] - ref_lse[:, seen]).abs().max().item() < 1e-5


PADDED_CASES = [
    # B, Hq, Hkv, Nq, Nk, d, q ranges, k ranges
    (3, 2, 2, 100, 100, 64, [(0, 100), (30, 100), (0, 57)], [(0, 100), (30, 100), (0, 57)]),
    (2, 4, 1, 1, 300, 128, [(0, 1), (0, 1)], [(44, 300), (0, 129)]),
    (2, 4, 2, 130, 260, 64, [(0, 130), (5, 130)], [(10, 250), (0, 260)]),
]


def _padded_inputs(B, Hq, Hkv, Nq, Nk, d, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Nq, d, generator=g).half()
    k = torch.randn(B, Hkv, Nk, d, generator=g).half()
    v = torch.randn(B, Hkv, Nk, d, generator=g).half()
    return q, k, v


def padded_mask(B, Nq, Nk, qr, kr, mode):
    """[B, 1, Nq, Nk] boolean mask of a padded batch (as an HF model builds it)."""
    i = torch.arange(Nq)[:, None]
    j = torch.arange(Nk)[None, :]
    base = torch.ones(Nq, Nk, dtype=torch.bool)
    if mode:
        base = j <= i + orc.kvcache_offset(Nq, Nk, mode)
    mask = torch.zeros(B, 1, Nq, Nk, dtype=torch.bool)
    for b in range(B):
        keys = (j >= kr[b][0]) & (j < kr[b][1])
        rows = (i >= qr[b][0]) & (i < qr[b][1])
        mask[b, 0] = base & keys & rows
    return mask


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", PADDED_CASES, ids=[str(c[:6]) for c in PADDED_CASES])
def test_padded_oracle_matches_torch_sdpa(case, mode):
    B, Hq, Hkv, Nq, Nk, d, qr, kr = case
    q, k, v = _padded_inputs(B, Hq, Hkv, Nq, Nk, d, seed=Nq + Nk + mode)
    o, lse = orc.attention_padded_fp32(q, k, v, [a for a, _ in qr], [b for _, b in qr],
                                       [a for a, _ in kr], [b for _, b in kr], causal_mode=mode)
    mask = padded_mask(B, Nq, Nk, qr, kr, mode)
    G = Hq // Hkv
    kx = k.repeat_interleave(G, dim=1).float()
    vx = v.repeat_interleave(G, dim=1).float()
    ref = F.scaled_dot_product_attention(q.float(), kx, vx, attn_mask=mask)
    seen = mask[:, 0].any(dim=-1)[:, None, :].expand(B, Hq, Nq)
    assert (o[seen] - ref[seen]).abs().max().item() < 1e-5
    assert (o[~seen] == 0).all() and torch.isinf(lse[~seen]).all()


def test_varlen_and_padded_argument_errors():
    lib = abi.load()
    n = abi.ctypes.c_void_p(0)
    # head_dim 96 -> FA_ERR_UNSUPPORTED_HEAD_DIM; dtype 7 -> FA_ERR_DTYPE;
    # negative total -> FA_ERR_INVALID_ARG; Hq % Hkv -> FA_ERR_GQA_DIVISIBILITY
    assert lib.fa_fwd_varlen(n, n, n, n, n, n, n, 1, 2, 2, 4, 4, 4, 4, 96, 0.1, 0, 0, n) == 2
    assert lib.fa_fwd_varlen(n, n, n, n, n, n, n, 1, 2, 2, 4, 4, 4, 4, 64, 0.1, 0, 7, n) == 5
    assert lib.fa_fwd_varlen(n, n, n, n, n, n, n, 1, 2, 2, -1, 4, 4, 4, 64, 0.1, 0, 0, n) == 1
    assert lib.fa_fwd_varlen(n, n, n, n, n, n, n, 1, 3, 2, 4, 4, 4, 4, 64, 0.1, 0, 0, n) == 3
    assert lib.fa_fwd_varlen(n, n, n, n, n, n, n, 1, 2, 2, 4, 4, 4, 4, 64, 0.1, 3, 0, n) == 1
    # empty problems are no-ops
    assert lib.fa_fwd_varlen(n, n, n, n, n, n, n, 0, 2, 2, 0, 0, 0, 0, 64, 0.1, 0, 0, n) == 0
    assert lib.fa_fwd_padded(n, n, n, n, n, n, n, n, n, 2, 2, 2, 8, 8, 128, 0.1, 0, 9, n) == 5
    assert lib.fa_fwd_padded(n, n, n, n, n, n, n, n, n, 2, 4, 3, 8, 8, 128, 0.1, 0, 0, n) == 3
    assert lib.fa_fwd_padded(n, n, n, n, n, n, n, n, n, 0, 2, 2, 8, 8, 128, 0.1, 0, 0, n) == 0


def test_python_api_argument_errors():
    import flash_attention_sm75 as fa
    q = torch.zeros(8, 2, 64, dtype=torch.float16)
    with pytest.raises(ValueError):
        fa.flash_attention_varlen_forward(q[None], q, q, [0, 8], [0, 8], 8, 8)
    with pytest.raises(RuntimeError):
        fa.flash_attention_varlen_forward(torch.zeros(8, 2, 96), q, q, [0, 8], [0, 8], 8, 8)
    with pytest.raises(ValueError):
        fa.flash_attention_varlen_forward(q, q, q, [0, 8], [0, 8], 8, 8, causal=True,
                                          causal_alignment="middle")
    Q = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    with pytest.raises(ValueError):
        fa.flash_attention_forward_padded(Q[0], Q, Q, [0], [8], [0], [8])
