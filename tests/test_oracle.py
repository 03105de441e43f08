"""The oracle against the reference's own outputs (golden fixtures) — CPU only."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as orc

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "golden_*.npz")))


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 10


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[7:-4] for p in GOLDEN])
def test_oracle_matches_reference_golden(path):
    z = np.load(path)
    q, k, v = (torch.from_numpy(z[n]) for n in ("q", "k", "v"))
    causal, scale = bool(z["causal"]), float(z["scale"])
    ref = torch.from_numpy(z["o_ref"])
    # restated reference (after the restated GQA expansion) — same torch ops, same bits
    ke, ve = orc.expand_kv_for_gqa(q.size(1), k, v)
    o16 = orc.attention_reference(q, ke, ve, causal=causal, scale=scale)
    assert torch.equal(o16, ref) or (o16.float() - ref.float()).abs().max().item() <= 1e-3
    # chunked fp32 oracle with native GQA mapping: within one fp16 rounding of the reference
    o32, lse = orc.attention_fp32(q, k, v, causal=causal, scale=scale, key_chunk=48)
    assert (o32 - ref.float()).abs().max().item() <= 2e-3
    assert torch.isfinite(lse).all()


def test_lse_matches_logsumexp():
    cfg = orc.AttnConfig("t", 2, 4, 2, 200, 64, True)
    q, k, v = orc.make_inputs(cfg, seed=3)
    o, lse = orc.attention_fp32(q, k, v, causal=True, key_chunk=64)
    ke, ve = orc.expand_kv_for_gqa(4, k, v)
    s = q.float() @ ke.float().transpose(-1, -2) / 8.0
    s.masked_fill_(torch.triu(torch.ones(200, 200, dtype=torch.bool), 1), float("-inf"))
    assert (lse - torch.logsumexp(s, -1)).abs().max().item() < 1e-5
    assert (o - torch.softmax(s, -1) @ ve.float()).abs().max().item() < 1e-5


def test_row_sampling_equals_full():
    cfg = orc.AttnConfig("t", 1, 2, 2, 300, 128, True)
    q, k, v = orc.make_inputs(cfg, seed=5)
    rows = orc.sample_rows(300, 20, seed=1)
    assert rows[0].item() == 0 and rows[-1].item() == 299
    o_all, l_all = orc.attention_fp32(q, k, v, causal=True)
    o_s, l_s = orc.attention_fp32(q, k, v, causal=True, rows=rows, key_chunk=100)
    assert torch.allclose(o_all[:, :, rows], o_s, atol=1e-5)
    assert torch.allclose(l_all[:, :, rows], l_s, atol=1e-5)


def test_gqa_mapping_is_repeat_interleave():
    k = torch.arange(2 * 3 * 1 * 1, dtype=torch.float32).reshape(2, 3, 1, 1)
    ke, _ = orc.expand_kv_for_gqa(6, k, k)
    # query head h reads kv head h // 2
    assert ke[0, :, 0, 0].tolist() == [0, 0, 1, 1, 2, 2]
    with pytest.raises(RuntimeError, match="not divisible"):
        orc.expand_kv_for_gqa(5, k, k)


def test_inputs_deterministic_and_shaped():
    for name, cfg in orc.CONFIGS.items():
        if cfg.N > 2048:
            continue
        a = orc.make_inputs(cfg, seed=7)
        b = orc.make_inputs(cfg, seed=7)
        assert all(torch.equal(x, y) for x, y in zip(a, b))
        assert a[0].shape == (cfg.B, cfg.Hq, cfg.N, cfg.d)
        assert a[1].shape == (cfg.B, cfg.Hkv, cfg.N, cfg.d)


def test_outlier_rows_scaled():
    cfg = orc.AttnConfig("t", 1, 1, 1, 1000, 64, False, k_outlier_frac=0.01)
    plain = orc.AttnConfig("t", 1, 1, 1, 1000, 64, False)
    _, k1, _ = orc.make_inputs(cfg, seed=1)
    _, k0, _ = orc.make_inputs(plain, seed=1)
    changed = (k1 != k0).any(-1).sum().item()
    assert changed == 10


def test_flop_and_byte_counts():
    c = orc.CONFIGS
    assert c["c2"].flops == pytest.approx(1.2885e10, rel=1e-3)
    assert c["c3"].flops == pytest.approx(1.7180e10, rel=1e-3)
    assert c["c4"].flops == pytest.approx(2.7488e11, rel=1e-3)
    assert c["c5"].flops == pytest.approx(4.3980e12, rel=1e-3)
    assert c["c5c"].flops == pytest.approx(2.1990e12, rel=1e-3)
    assert c["c1"].min_bytes == 264192
    assert c["c4"].min_bytes == 168820736


def test_check_metrics():
    ref = torch.tensor([1.0, -2.0, 0.0])
    assert orc.check(ref.half(), ref)["ok"]
    bad = ref + torch.tensor([0.0, 0.0, 0.01])
    r = orc.check(bad, ref)
    assert not r["ok"] and r["max_abs_err"] == pytest.approx(0.01)
    assert not orc.check(torch.tensor([float("nan"), 0, 0]), ref)["ok"]
