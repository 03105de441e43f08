"""fa_naive_fwd_noalloc: the materialised attention without any device
allocation, for callers that cannot allocate while they run (closed allocators,
real-time loops, runtimes that own all device memory).  Its scores live in a
16 MiB file-scope device array shared by all calls on a device.

Checked through the C ABI against the allocating entry point fa_naive_fwd
(same kernels, caller-provided workspace) on two calls in a row with
different shapes, within the tests' tolerance (2e-3 + 1e-2*|ref|), and
against the CPU oracle.  This file is collected last so that a run stopping
at the first failure has already run every other test."""
import math

import pytest
import torch

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _run_both(lib, B, H, N, d, causal, seed):
    cfg = orc.AttnConfig("t", B, H, H, N, d, causal)
    q, k, v = orc.make_inputs(cfg, seed=seed)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    scale = 1.0 / math.sqrt(d)
    stream = abi.stream_ptr()
    o_alloc = torch.empty_like(qd)
    ws = torch.empty(B * H * N * N, dtype=torch.float32, device="cuda")
    rc = lib.fa_naive_fwd(abi.ptr(qd), abi.ptr(kd), abi.ptr(vd), abi.ptr(o_alloc), B, H, N, d,
                          scale, int(causal), abi.ptr(ws), stream)
    assert rc == 0
    o_static = torch.full_like(qd, float("nan"))
    rc = lib.fa_naive_fwd_noalloc(abi.ptr(qd), abi.ptr(kd), abi.ptr(vd), abi.ptr(o_static), B, H, N,
                                  d, scale, int(causal), stream)
    assert rc == 0, lib.fa_error_string(rc)
    torch.cuda.synchronize()
    a, b = o_alloc.float().cpu(), o_static.float().cpu()
    assert torch.isfinite(b).all()
    assert ((a - b).abs() <= ATOL + RTOL * a.abs()).all()
    ref, _ = orc.attention_fp32(q, k, v, causal=causal, scale=scale)
    assert orc.check(o_static.cpu(), ref)["ok"]


def test_noalloc_matches_allocating_entry_point_twice(sm100):
    lib = abi.load()
    # two calls in a row: the second reuses the array left by the first
    _run_both(lib, 2, 3, 200, 64, True, seed=11)
    _run_both(lib, 1, 4, 256, 128, False, seed=12)


def test_noalloc_rejects_sizes_beyond_its_scratch(sm100):
    lib = abi.load()
    o = torch.full((1, 1, 2049, 64), 5.0, dtype=torch.float16, device="cuda")
    q = torch.zeros_like(o)
    # 1 * 1 * 2049^2 > 4Mi floats
    rc = lib.fa_naive_fwd_noalloc(abi.ptr(q), abi.ptr(q), abi.ptr(q), abi.ptr(o), 1, 1, 2049, 64,
                                  0.125, 0, abi.stream_ptr())
    assert rc == 11
    assert b"scratch" in lib.fa_error_string(rc)
    torch.cuda.synchronize()
    assert torch.all(o == 5.0)  # nothing was launched
