"""The reference's own PyTorch binding (src/bindings/pytorch_extension.cpp),
compiled unchanged and linked against lib/libfa_b200.so in place of the
reference's two sm_75 kernel files (recipe: oracle/build_ref_binding.py,
output oracle/_ref/), loads and runs: proof that the C ABI is a drop-in for
the reference's launchers.  The module shares its name with this repo's
binding, so each check runs in a separate process (tests/ref_binding_check.py).
"""
import glob
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _built():
    return glob.glob(os.path.join(REPO, "oracle", "_ref", "flash_attn_sm75_cuda*.so"))


def _run(mode):
    if not _built():
        pytest.skip("oracle/_ref holds no reference binding (built only where the reference "
                    "checkout is present: python oracle/build_ref_binding.py <root>)")
    r = subprocess.run([sys.executable, os.path.join(HERE, "ref_binding_check.py"), mode],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_reference_binding_loads_and_exports_its_four_functions():
    out = _run("names")
    assert out["module"].startswith(os.path.join("oracle", "_ref"))
    assert out["names"] == ["naive_attention_forward", "flash_attention_forward",
                            "flash_attention_forward_scalar", "flash_attention_forward_wmma_qk"]


@pytest.mark.gpu
def test_reference_binding_runs_the_reference_d128_flow(sm100):
    out = _run("gpu")
    bad = [c for c in out["cases"] if not c["ok"]]
    assert out["all_ok"], bad
    assert out["fp32_rejected"]
    assert len(out["cases"]) >= 20
