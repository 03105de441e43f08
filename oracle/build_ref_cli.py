"""Builds the REFERENCE's own standalone benchmark CLIs, unchanged, for the
B200 — the same-box comparison column of the reference's sm_75 kernels.

The reference's two standalone tools, flash_mha_flatargs (full attention) and
flash_mha_v2 (full + causal), are single CUDA files
(flash-attention-sm75-fused/src/flash_mha_flatargs.cu, flash_mha_v2.cu) that
include only the reference's own headers (flash-attention-sm75-fused/include)
and use WMMA fragments, which sm_100a still executes.  This recipe compiles
them where they lie in the reference checkout with nvcc for sm_100a into
``oracle/_ref/`` (git-ignored; it travels to the GPU box with the tree), as
``flash_mha_flatargs_ref`` and ``flash_mha_v2_ref``.  Only ``bench.py`` (its
``reference_sm75`` comparison column) and the GPU tests run them; they are
never on this repository's product path.

    python oracle/build_ref_cli.py <reference checkout root> [--force]
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
TOOLS = ("flash_mha_flatargs", "flash_mha_v2")


def out_path(tool):
    return os.path.join(OUT_DIR, tool + "_ref")


def build(ref_root, force=False, verbose=False):
    """Compile both CLIs into oracle/_ref/; returns their paths, or None when
    the reference checkout is absent."""
    base = os.path.join(ref_root, "flash-attention-sm75-fused")
    srcs = [os.path.join(base, "src", t + ".cu") for t in TOOLS]
    if not all(os.path.exists(s) for s in srcs):
        return None
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    outs = []
    for tool, src in zip(TOOLS, srcs):
        out = out_path(tool)
        outs.append(out)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
            continue
        cmd = [nvcc, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
               "-I", os.path.join(base, "include"), src, "-o", out]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"reference CLI build failed: {tool}")
    return outs


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit(__doc__)
    paths = build(sys.argv[1], force="--force" in sys.argv, verbose=True)
    print(paths if paths else "reference checkout not found")
