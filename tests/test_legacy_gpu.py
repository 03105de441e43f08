"""The reference-compatible C entry points (blocking launchers, standalone
launchers) and the two command-line tools, on the GPU."""
import ctypes
import math
import os
import re
import subprocess

import pytest
import torch

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu

BIN = os.path.join(abi.PKG_DIR, "lib")


def _inputs(B, H, N, d, causal, seed=1):
    return orc.make_inputs(orc.AttnConfig("t", B, H, H, N, d, causal), seed=seed)


@pytest.mark.parametrize("name,d", [("launch_flash_attention_forward", 64),
                                    ("launch_flash_attention_forward", 128),
                                    ("launch_flash_attention_forward_scalar", 64),
                                    ("launch_flash_attention_forward_wmma_qk", 64)])
@pytest.mark.parametrize("causal", [False, True])
def test_blocking_launchers(sm100, name, d, causal):
    q, k, v = _inputs(2, 4, 200, d, causal)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = torch.zeros_like(qd)
    torch.cuda.synchronize()
    getattr(abi.load(), name)(abi.ptr(qd), abi.ptr(kd), abi.ptr(vd), abi.ptr(o), 2, 4, 200, d,
                              1.0 / math.sqrt(d), causal)
    ref, _ = orc.attention_fp32(q, k, v, causal=causal)
    assert orc.check(o.cpu(), ref)["ok"]


def test_blocking_launcher_rejects_head_dim(sm100, capfd):
    q = torch.zeros(1, 1, 16, 128, dtype=torch.float16, device="cuda")
    o = torch.full_like(q, 7.0)
    abi.load().launch_flash_attention_forward_scalar(abi.ptr(q), abi.ptr(q), abi.ptr(q), abi.ptr(o),
                                                     1, 1, 16, 128, 1.0, False)
    assert "head_dim=128 not supported" in capfd.readouterr().err
    assert torch.all(o == 7.0)  # nothing was launched


def test_naive_launcher_with_workspace(sm100):
    q, k, v = _inputs(1, 2, 96, 64, True)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = torch.empty_like(qd)
    ws = torch.empty(1 * 2 * 96 * 96, dtype=torch.float32, device="cuda")
    abi.load().launch_naive_attention(abi.ptr(qd), abi.ptr(kd), abi.ptr(vd), abi.ptr(o), 1, 2, 96,
                                      64, 0.125, True, abi.ptr(ws))
    ref, _ = orc.attention_fp32(q, k, v, causal=True, scale=0.125)
    assert orc.check(o.cpu(), ref)["ok"]


@pytest.mark.parametrize("mode", [0, 1])
def test_standalone_launchers(sm100, mode):
    q, k, v = _inputs(2, 3, 160, 64, bool(mode))
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    o = torch.empty_like(qd)
    lib = abi.load()
    if mode == 0:
        rc = lib.flatargs_launch(abi.ptr(qd), abi.ptr(kd), abi.ptr(vd), abi.ptr(o), 2, 3, 160, 0.125,
                                 abi.stream_ptr())
    else:
        rc = lib.launch_v2(abi.ptr(qd), abi.ptr(kd), abi.ptr(vd), abi.ptr(o), 2, 3, 160, 0.125, 1,
                           abi.stream_ptr())
    assert rc == 0
    torch.cuda.synchronize()
    ref, _ = orc.attention_fp32(q, k, v, causal=bool(mode), scale=0.125)
    assert orc.check(o.cpu(), ref)["ok"]


def _run(tool, *args):
    out = subprocess.run([os.path.join(BIN, tool), *map(str, args)], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    return out.stdout


def test_cli_flatargs_output_contract(sm100):
    text = _run("flash_mha_flatargs", 1, 4, 128, 3, 10)
    assert "PASS" in text and "FAIL" not in text
    # regex of the reference's benchmark_sdpa_final.py:116-123
    m = re.search(r"\bms\b\s+([\d.]+)\s+([\d.]+)\s+([\d.]+)", text)
    assert m and 0 < float(m.group(1)) <= float(m.group(2)) <= float(m.group(3))


def test_cli_v2_output_contract(sm100):
    text = _run("flash_mha_v2", 2, 2, 200, 3, 10)
    assert text.count("PASS") == 2 and "FAIL" not in text
    # regexes of the reference's benchmark_sdpa_final.py:126-141
    full = re.search(r"^FULL\s+([\d.]+)\s+([\d.]+)\s+([\d.]+)", text, re.MULTILINE)
    causal = re.search(r"^CAUSAL\s+([\d.]+)\s+([\d.]+)\s+([\d.]+)", text, re.MULTILINE)
    assert full and causal


def test_cli_headline_shape_runs(sm100):
    text = _run("flash_mha_flatargs", 4, 12, 1024, 3, 20)
    m = re.search(r"\bms\b\s+([\d.]+)\s+([\d.]+)\s+([\d.]+)", text)
    assert m and float(m.group(2)) < 1.0
