"""Backward oracle on the CPU: autograd through the fp32 attention
(attention_ref.py restated) agrees with the FlashAttention-2 backward formulas
that the sm_100a kernels implement."""
import pytest
import torch

from oracle import attention_oracle as orc


@pytest.mark.parametrize("B,Hq,Hkv,N,d,causal", [
    (1, 2, 2, 37, 64, False), (1, 4, 2, 64, 64, True), (2, 6, 3, 50, 128, True),
    (1, 2, 1, 16, 128, False)])
def test_oracle_grads_match_fa2_formulas(B, Hq, Hkv, N, d, causal):
    g = torch.Generator().manual_seed(N + d)
    q = torch.randn(B, Hq, N, d, generator=g).half()
    k = torch.randn(B, Hkv, N, d, generator=g).half()
    v = torch.randn(B, Hkv, N, d, generator=g).half()
    do = torch.randn(B, Hq, N, d, generator=g).half()
    a = orc.attention_grads_fp32(q, k, v, do, causal=causal)
    b = orc.attention_grads_formulas(q, k, v, do, causal=causal)
    for x, y in zip(a, b):
        assert (x - y).abs().max().item() < 1e-4
