"""Parity of fa_fwd_kvcache (Nq != Nk: decode, chunked prefill) against the CPU
oracle, through the C ABI.

Tolerance as for fa_fwd: |O - O_ref| <= 2e-3 + 1e-2*|O_ref| (fp16; bf16
1.6e-2 + 2e-2*|ref|), LSE within 1e-4.  Covers GQA row packing (Nq <= 128),
split-KV with the combine kernel (workspace given) and without (workspace
None), both causal alignments, ragged Nk, and rows that see no key.
"""
import pytest
import torch

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu

BF16_ATOL, BF16_RTOL = 1.6e-2, 2e-2


def _inputs(B, Hq, Hkv, Nq, Nk, d, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Nq, d, generator=g).to(dtype)
    k = torch.randn(B, Hkv, Nk, d, generator=g).to(dtype)
    v = torch.randn(B, Hkv, Nk, d, generator=g).to(dtype)
    return q, k, v


def run(q, k, v, mode, workspace=True):
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    rc = abi.fa_fwd_kvcache(q, k, v, o, lse, causal=mode, workspace=workspace)
    assert rc == 0, abi.load().fa_error_string(rc)
    torch.cuda.synchronize()
    assert abi.load().fa_device_status(1) == 0
    return o, lse


def parity(B, Hq, Hkv, Nq, Nk, d, mode, seed=0, dtype=torch.float16, workspace=True):
    q, k, v = _inputs(B, Hq, Hkv, Nq, Nk, d, seed, dtype)
    o, lse = run(q.cuda(), k.cuda(), v.cuda(), mode, workspace)
    ref_o, ref_lse = orc.attention_fp32(q, k, v, causal=mode != 0,
                                        causal_offset=orc.kvcache_offset(Nq, Nk, mode))
    o, lse = o.cpu(), lse.cpu()
    if dtype == torch.bfloat16:
        r = orc.check(o, ref_o, atol=BF16_ATOL, rtol=BF16_RTOL)
    else:
        r = orc.check(o, ref_o)
    assert r["ok"], r
    finite = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), finite)
    assert orc.check_lse(lse[finite], ref_lse[finite])["ok"]
    return o, lse


DECODE = [
    # B, Hq, Hkv, Nq, Nk, d
    (1, 32, 8, 1, 4096, 128),   # GQA 4: packed, split
    (4, 8, 1, 1, 1000, 128),    # MQA 8, ragged Nk
    (2, 16, 16, 1, 2048, 64),   # MHA decode
    (1, 8, 2, 1, 77, 64),       # single ragged tile
    (1, 4, 4, 1, 1, 128),       # one key
]


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("case", DECODE, ids=[str(c) for c in DECODE])
def test_decode(sm100, case, mode):
    parity(*case, mode=mode, seed=sum(case))


CHUNKED = [
    (1, 8, 2, 7, 300, 128),     # packed rows (G*Nq = 28)
    (2, 4, 1, 32, 1024, 64),    # packed, G*Nq = 128
    (1, 4, 2, 96, 640, 128),    # packed, G*Nq = 192 (two tiles)
    (1, 4, 2, 129, 700, 128),   # unpacked (Nq > 128)
    (1, 2, 2, 300, 1000, 64),   # MHA chunk
    (1, 8, 8, 256, 256, 128),   # square: same as fa_fwd
]


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", CHUNKED, ids=[str(c) for c in CHUNKED])
def test_chunked_prefill(sm100, case, mode):
    parity(*case, mode=mode, seed=sum(case) + mode)


def test_rows_without_keys(sm100):
    """Bottom-right with Nq > Nk: the first rows see nothing -> O = 0, LSE = -inf."""
    o, lse = parity(1, 4, 2, 200, 72, 128, mode=1, seed=5)
    assert torch.equal(o[:, :, :128], torch.zeros_like(o[:, :, :128]))


def test_bf16_decode_and_chunk(sm100):
    parity(2, 16, 4, 1, 3000, 128, mode=0, seed=1, dtype=torch.bfloat16)
    parity(1, 8, 2, 50, 600, 64, mode=1, seed=2, dtype=torch.bfloat16)


@pytest.mark.parametrize("case", [(1, 32, 8, 1, 8192, 128), (1, 8, 2, 16, 4096, 64)])
def test_split_matches_unsplit(sm100, case):
    """The split-KV path (workspace) and the single-CTA path agree to rounding."""
    q, k, v = (t.cuda() for t in _inputs(*case, seed=11))
    lib = abi.load()
    assert lib.fa_fwd_kvcache_workspace_bytes(*case) > 0  # this shape is split
    o1, l1 = run(q, k, v, 0, workspace=True)
    o2, l2 = run(q, k, v, 0, workspace=None)
    assert (o1.float() - o2.float()).abs().max().item() <= 2e-3
    assert (l1 - l2).abs().max().item() <= 1e-4


def test_square_matches_fa_fwd_bitwise(sm100):
    """Nq == Nk > 128 runs the same tiles as fa_fwd."""
    q, k, v = (t.cuda() for t in _inputs(2, 8, 2, 384, 384, 128, seed=4))
    o1, l1 = run(q, k, v, 1, workspace=None)
    o2 = torch.empty_like(q)
    l2 = torch.empty_like(l1)
    assert abi.fa_fwd(q, k, v, o2, l2, causal=True) == 0
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_small_workspace_runs_unsplit(sm100):
    q, k, v = (t.cuda() for t in _inputs(1, 32, 8, 1, 4096, 128, seed=6))
    tiny = torch.empty(64, dtype=torch.uint8, device="cuda")
    o1, l1 = run(q, k, v, 0, workspace=tiny)
    o2, l2 = run(q, k, v, 0, workspace=None)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


# Query blocks of at most 16 rows per (batch, KV head) run the decode kernel
# (keys on the MMA's M dimension); 17 rows and more the attention kernel.
DECODE_BLOCKS = [
    # B, Hq, Hkv, Nq, Nk, d
    (2, 16, 2, 2, 3000, 128),   # GQA 8 x 2 tokens = 16 rows
    (1, 12, 4, 4, 900, 64),     # GQA 3 x 4 tokens = 12 rows
    (3, 4, 4, 16, 2000, 128),   # MHA, 16 tokens
    (1, 6, 2, 5, 128, 128),     # 15 rows, exactly one K/V tile
    (2, 8, 8, 3, 50, 64),       # Nk below one tile
    (2, 16, 2, 1, 1500, 64),    # 8 rows at d = 64: two warpgroups x two key halves
    (1, 6, 1, 1, 777, 64),      # 6 of 8 rows: the second warpgroup's last rows are past the block
    (1, 10, 1, 1, 300, 128),    # 10 of 16 rows: four warpgroups, the last one empty
    (1, 17, 1, 1, 500, 64),     # 17 rows: the attention kernel
]


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("case", DECODE_BLOCKS, ids=[str(c) for c in DECODE_BLOCKS])
@pytest.mark.parametrize("workspace", [True, None], ids=["split", "unsplit"])
def test_decode_blocks(sm100, case, mode, workspace):
    parity(*case, mode=mode, seed=sum(case) + mode, workspace=workspace)


def test_decode_blocks_bf16(sm100):
    parity(2, 16, 2, 2, 3000, 128, mode=1, seed=3, dtype=torch.bfloat16)
    parity(1, 12, 4, 4, 900, 64, mode=2, seed=4, dtype=torch.bfloat16)


def test_decode_many_items_per_cta(sm100):
    """Enough (head, split) items that every persistent CTA walks several,
    carrying the K/V ring, the Q double buffer and the deferred epilogue over
    item boundaries; split and unsplit results agree to rounding."""
    q, k, v = (t.cuda() for t in _inputs(16, 32, 8, 1, 4096, 128, seed=12))
    o1, l1 = run(q, k, v, 0, workspace=True)
    o2, l2 = run(q, k, v, 0, workspace=None)
    ref_o, ref_lse = orc.attention_fp32(q.cpu()[:2], k.cpu()[:2], v.cpu()[:2])
    assert orc.check(o1.cpu()[:2], ref_o)["ok"]
    assert orc.check_lse(l1.cpu()[:2], ref_lse)["ok"]
    assert (o1.float() - o2.float()).abs().max().item() <= 2e-3
    assert (l1 - l2).abs().max().item() <= 1e-4
