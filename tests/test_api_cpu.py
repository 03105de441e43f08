"""Python API behaviour that needs no GPU: argument checks and error types of
flash_attention_sm75 (reference src/flash_attention_sm75/ops.py, tests/test_api.py)."""
import pytest
import torch

import flash_attention_sm75 as fa
from flash_attention_sm75 import ops


def test_public_surface():
    # the reference's surface (src/flash_attention_sm75/__init__.py:1-4) plus additions
    assert fa.__all__ == ["flash_attention_forward", "flash_attention_forward_kvcache",
                          "flash_attention_forward_host", "flash_attention_varlen_forward",
                          "flash_attention_forward_padded", "flash_attention",
                          "flash_attention_padded", "flash_attention_varlen"]
    assert isinstance(fa.__version__, str)


def test_kvcache_argument_errors():
    q = torch.zeros(1, 4, 1, 64, dtype=torch.float16)
    k = torch.zeros(1, 2, 16, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="4D"):
        fa.flash_attention_forward_kvcache(q[0], k, k)
    with pytest.raises(RuntimeError, match="supports head_dim=64 or 128"):
        fa.flash_attention_forward_kvcache(torch.zeros(1, 4, 1, 96), k, k)
    with pytest.raises(ValueError, match="causal_alignment"):
        fa.flash_attention_forward_kvcache(q, k, k, causal=True, causal_alignment="middle")
    with pytest.raises(RuntimeError, match="not divisible"):
        fa.flash_attention_forward_kvcache(torch.zeros(1, 3, 1, 64), k, k)
    with pytest.raises(RuntimeError, match="CUDA"):
        fa.flash_attention_forward_kvcache(q, k, k)  # CPU tensors are rejected by the binding


def test_rejects_non_4d():
    q = torch.zeros(8, 128, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="Q must be 4D"):
        fa.flash_attention_forward(q, q, q)


def test_rejects_head_dim_96_with_reference_message():
    q = torch.zeros(1, 8, 128, 96, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="supports head_dim=64 or 128"):
        fa.flash_attention_forward(q, q, q)


def test_gqa_divisibility_error():
    q = torch.zeros(1, 6, 16, 64, dtype=torch.float16)
    k = torch.zeros(1, 4, 16, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="not divisible"):
        fa.flash_attention_forward(q, k, k)


def test_cpu_tensors_fail_loudly_no_fallback():
    q = torch.zeros(1, 2, 16, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        fa.flash_attention_forward(q, q, q)


def test_backward_raises_not_implemented_with_both_message_forms():
    with pytest.raises(NotImplementedError) as e:
        ops.FlashAttentionSM75Function.backward(None, None)
    msg = str(e.value)
    assert "Backward pass not implemented" in msg          # reference ops.py:49-51
    assert "Backward pass is not implemented" in msg       # reference tests/test_api.py:38


def test_expand_kv_helper_matches_repeat_interleave():
    q = torch.zeros(1, 8, 4, 64)
    k = torch.arange(2 * 4 * 64, dtype=torch.float32).reshape(1, 2, 4, 64)
    ke, ve = ops._expand_kv_for_gqa(q, k, k)
    assert ke.shape == (1, 8, 4, 64)
    assert torch.equal(ke[0, 3], k[0, 0]) and torch.equal(ke[0, 4], k[0, 1])


def test_extension_module_binds_reference_names():
    import flash_attn_sm75_cuda as C
    for name in ("naive_attention_forward", "flash_attention_forward",
                 "flash_attention_forward_scalar", "flash_attention_forward_wmma_qk",
                 "flash_attention_forward_lse", "device_status"):
        assert hasattr(C, name)


def test_host_api_argument_errors():
    q = torch.zeros(1, 4, 16, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="4D"):
        fa.flash_attention_forward_host(q[0], q, q)
    with pytest.raises(RuntimeError, match="supports head_dim=64 or 128"):
        x = torch.zeros(1, 4, 16, 96, dtype=torch.float16)
        fa.flash_attention_forward_host(x, x, x)
    with pytest.raises(RuntimeError, match="not divisible"):
        fa.flash_attention_forward_host(q, q[:, :3], q[:, :3])
    with pytest.raises(ValueError, match="out must be"):
        fa.flash_attention_forward_host(q, q, q, out=torch.zeros(1, 4, 16, 32, dtype=torch.float16))
