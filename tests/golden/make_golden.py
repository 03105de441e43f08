"""Generate the golden fixtures in this folder from the REFERENCE implementation.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own CPU path — ``attention_reference`` from
src/reference/attention_ref.py and ``_expand_kv_for_gqa`` from
src/flash_attention_sm75/ops.py (its CUDA extension import is stubbed, only the
pure-torch helper is used) — on small seeded inputs and stores inputs and
outputs as ``golden_<case>.npz``.  Nothing at test time reads the reference.

Each case holds: q, k, v (fp16), o_ref (fp16 output of attention_reference,
after GQA expansion for GQA cases), plus scalars causal, scale.
"""
import os
import sys
import types

import numpy as np
import torch

CASES = [
    # name, B, Hq, Hkv, N, d, causal, seed
    ("full_d64_n64", 1, 2, 2, 64, 64, False, 1),
    ("causal_d64_n64", 1, 2, 2, 64, 64, True, 2),
    ("full_d64_n17", 1, 2, 2, 17, 64, False, 3),
    ("causal_d64_n1", 1, 1, 1, 1, 64, True, 4),
    ("causal_d64_n16", 1, 2, 2, 16, 64, True, 5),
    ("full_d128_n100", 1, 1, 1, 100, 128, False, 6),
    ("causal_d128_n129", 1, 1, 1, 129, 128, True, 7),
    ("full_d64_n256_b2", 2, 2, 2, 256, 64, False, 8),
    ("causal_d128_n300", 1, 2, 2, 300, 128, True, 9),
    ("gqa_causal_d128_n96", 1, 4, 2, 96, 128, True, 10),
    ("gqa_full_d64_n130", 2, 4, 1, 130, 64, False, 11),
]


def main(ref_root):
    sys.path.insert(0, os.path.join(ref_root, "src"))
    from reference.attention_ref import attention_reference  # noqa: E402

    # ops.py imports the compiled extension at module load; a stub lets us
    # import the pure-torch GQA helper without it.
    sys.modules.setdefault("flash_attn_sm75_cuda", types.ModuleType("flash_attn_sm75_cuda"))
    from flash_attention_sm75.ops import _expand_kv_for_gqa  # noqa: E402

    out_dir = os.path.dirname(os.path.abspath(__file__))
    for name, B, Hq, Hkv, N, d, causal, seed in CASES:
        torch.manual_seed(seed)
        q = torch.randn(B, Hq, N, d, dtype=torch.float16)
        k = torch.randn(B, Hkv, N, d, dtype=torch.float16)
        v = torch.randn(B, Hkv, N, d, dtype=torch.float16)
        scale = 1.0 / float(np.sqrt(d))
        ke, ve = _expand_kv_for_gqa(q, k, v)
        o = attention_reference(q, ke, ve, causal=causal, scale=scale)
        np.savez_compressed(
            os.path.join(out_dir, f"golden_{name}.npz"),
            q=q.numpy(), k=k.numpy(), v=v.numpy(), o_ref=o.numpy(),
            causal=np.array(causal), scale=np.array(scale, dtype=np.float64))
        print(name, tuple(q.shape), tuple(k.shape), "->", tuple(o.shape))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout root>")
    main(sys.argv[1])
