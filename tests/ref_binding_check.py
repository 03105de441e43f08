"""Run in a separate process by tests/test_reference_binding_*.py: imports the
reference's own binding (oracle/_ref/flash_attn_sm75_cuda*.so, compiled
unchanged from src/bindings/pytorch_extension.cpp and linked against
lib/libfa_b200.so) and, with a GPU, runs the reference's
tests/test_flash_d128.py:10-63 flow through it: seeded fp16 Q, K, V, the four
binding functions, results against the oracle.

    python tests/ref_binding_check.py names|gpu
Prints one JSON line.
"""
import json
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [os.path.join(REPO, "oracle", "_ref"), REPO]

import torch  # noqa: E402
import flash_attn_sm75_cuda as _C  # noqa: E402  (the reference's binding)

NAMES = ["naive_attention_forward", "flash_attention_forward", "flash_attention_forward_scalar",
         "flash_attention_forward_wmma_qk"]


def main(mode):
    out = {"module": os.path.relpath(_C.__file__, REPO),
           "names": [n for n in NAMES if hasattr(_C, n)]}
    if mode == "gpu":
        from oracle import attention_oracle as orc
        cases = [(1, 8, 128, 64, False), (1, 8, 512, 64, False), (1, 8, 1024, 64, True),
                 (1, 8, 128, 128, False), (1, 8, 256, 128, False), (2, 8, 256, 128, False),
                 (1, 16, 512, 128, False), (1, 8, 256, 128, True), (1, 8, 1024, 128, True),
                 (1, 2, 77, 128, True)]
        res = []
        for (B, H, N, d, causal) in cases:
            torch.manual_seed(42)
            q = torch.randn(B, H, N, d, dtype=torch.float16, device="cuda")
            k = torch.randn(B, H, N, d, dtype=torch.float16, device="cuda")
            v = torch.randn(B, H, N, d, dtype=torch.float16, device="cuda")
            scale = 1.0 / math.sqrt(d)
            ref, _ = orc.attention_fp32(q.cpu(), k.cpu(), v.cpu(), causal=causal, scale=scale)
            fns = ["flash_attention_forward"]
            if d == 64:
                fns += ["flash_attention_forward_scalar", "flash_attention_forward_wmma_qk"]
            if N <= 512:
                fns += ["naive_attention_forward"]
            for fn in fns:
                o = getattr(_C, fn)(q, k, v, causal, scale)
                torch.cuda.synchronize()
                r = orc.check(o.cpu(), ref)
                res.append({"case": [B, H, N, d, causal], "fn": fn, "ok": r["ok"],
                            "max_abs_err": r["max_abs_err"]})
        # the binding's own argument checks still fire (pytorch_extension.cpp:21-26)
        try:
            x = torch.zeros(1, 1, 16, 64, device="cuda")
            _C.flash_attention_forward(x, x, x, False, 1.0)
            fp32_rejected = False
        except RuntimeError as e:
            fp32_rejected = "must be FP16" in str(e)
        out.update({"cases": res, "all_ok": all(r["ok"] for r in res),
                    "fp32_rejected": fp32_rejected})
    print(json.dumps(out))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "names")
