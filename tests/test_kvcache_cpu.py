"""KV-cache / chunked-prefill extension (Nq != Nk), CPU side.

The oracle's generalisation (Nk keys, causal offset) is pinned against
PyTorch's own scaled_dot_product_attention on the CPU in fp32: bottom-right
alignment through an explicit mask, top-left through ``is_causal`` (SDPA's
rule for non-square inputs).  The C entry points are checked for their
argument errors and workspace query, which need no GPU.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

CASES = [
    # B, Hq, Hkv, Nq, Nk, d
    (1, 4, 1, 1, 300, 64),
    (2, 8, 2, 5, 129, 128),
    (1, 2, 2, 64, 200, 64),
    (1, 6, 3, 130, 257, 128),
    (1, 2, 1, 40, 40, 64),
]


def _inputs(B, Hq, Hkv, Nq, Nk, d, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Nq, d, generator=g).half()
    k = torch.randn(B, Hkv, Nk, d, generator=g).half()
    v = torch.randn(B, Hkv, Nk, d, generator=g).half()
    return q, k, v


def _sdpa(q, k, v, mode):
    Hq, Nq, Nk = q.size(1), q.size(2), k.size(2)
    kx = k.repeat_interleave(Hq // k.size(1), dim=1).float()
    vx = v.repeat_interleave(Hq // v.size(1), dim=1).float()
    if mode == 2:
        return F.scaled_dot_product_attention(q.float(), kx, vx, is_causal=True)
    mask = None
    if mode == 1:
        i = torch.arange(Nq)[:, None]
        j = torch.arange(Nk)[None, :]
        mask = j <= i + (Nk - Nq)
    return F.scaled_dot_product_attention(q.float(), kx, vx, attn_mask=mask)


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_oracle_matches_torch_sdpa(case, mode):
    B, Hq, Hkv, Nq, Nk, d = case
    q, k, v = _inputs(*case, seed=Nq * 7 + Nk + mode)
    off = orc.kvcache_offset(Nq, Nk, mode)
    o, lse = orc.attention_fp32(q, k, v, causal=mode != 0, causal_offset=off, key_chunk=100)
    ref = _sdpa(q, k, v, mode)
    assert (o - ref).abs().max().item() < 1e-5
    # LSE against a direct logsumexp with the same mask
    kx = k.repeat_interleave(Hq // Hkv, dim=1).float()
    s = q.float() @ kx.transpose(-1, -2) / math.sqrt(d)
    if mode:
        i = torch.arange(Nq)[:, None]
        j = torch.arange(Nk)[None, :]
        s = s.masked_fill(j > i + off, float("-inf"))
    assert (lse - torch.logsumexp(s, -1)).abs().max().item() < 1e-5


def test_oracle_rows_without_keys():
    """Bottom-right with Nq > Nk: the first Nq - Nk rows see no key."""
    q, k, v = _inputs(1, 2, 2, 10, 4, 64, seed=3)
    o, lse = orc.attention_fp32(q, k, v, causal=True, causal_offset=4 - 10)
    assert torch.equal(o[:, :, :6], torch.zeros_like(o[:, :, :6]))
    assert torch.isinf(lse[:, :, :6]).all() and (lse[:, :, :6] < 0).all()
    o2, _ = orc.attention_fp32(q[:, :, 6:], k, v, causal=True, causal_offset=0)
    assert (o[:, :, 6:] - o2).abs().max().item() < 1e-6


def test_kvcache_argument_errors_without_gpu():
    lib = abi.load()
    nul = abi.ptr(None)
    fake = abi.ctypes.c_void_p(1 << 20)
    call = lambda **kw: lib.fa_fwd_kvcache(*[kw.get(n, dflt) for n, dflt in (
        ("Q", fake), ("K", fake), ("V", fake), ("O", fake), ("lse", nul), ("B", 1), ("Hq", 4),
        ("Hkv", 2), ("Nq", 1), ("Nk", 64), ("d", 128), ("scale", 0.1), ("causal", 0),
        ("dtype", 0), ("ws", nul), ("wsb", 0), ("stream", nul))])
    # FA_ERR_* values from include/fa_b200.h
    assert call(d=96) == 2
    assert call(causal=3) == 1
    assert call(Hkv=3) == 3
    assert call(Nk=0) == 1
    assert call(Nq=-1) == 1
    assert call(dtype=7) == 5
    assert call(Q=nul) == 1
    assert call(Nq=0) == 0          # empty: nothing to do, no device needed
    assert call(B=0) == 0
    assert call(scale=float("inf")) == 1


def test_kvcache_workspace_query():
    lib = abi.load()
    # decode: few (batch*head, Q pair) units -> split, workspace > 0
    w = lib.fa_fwd_kvcache_workspace_bytes(1, 32, 8, 1, 8192, 128)
    assert w > 0
    # large prefill: enough units, no split
    assert lib.fa_fwd_kvcache_workspace_bytes(4, 32, 32, 8192, 8192, 128) == 0
    # invalid shapes ask for nothing
    assert lib.fa_fwd_kvcache_workspace_bytes(1, 6, 4, 1, 100, 128) == 0
    assert lib.fa_fwd_kvcache_workspace_bytes(1, 4, 4, 1, 100, 96) == 0
    # bytes = splits * rows * (d + 1) * 4: a whole number of rows per split
    rows = 1 * 8 * 4 * 1  # packed: Hkv heads x (G * Nq) rows
    assert w % (rows * (128 + 1) * 4) == 0
