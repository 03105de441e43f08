"""Builds the REFERENCE's own PyTorch binding, unchanged, against this repo's
C-ABI library — test infrastructure that proves the drop-in claim.

The reference links src/bindings/pytorch_extension.cpp with its two sm_75
kernel files into the module ``flash_attn_sm75_cuda`` (reference setup.py:10-25).
This recipe compiles that same binding source, read where it lies in the
reference checkout, with ``g++`` and links it against
``lib/libfa_b200.so`` in place of the two kernel files: the binding declares
the four ``launch_*`` launchers with ``half*`` arguments
(pytorch_extension.cpp:4-19) and the library exports them with ``void*``
arguments, the same C ABI.  The output goes to ``oracle/_ref/`` (git-ignored;
it travels to the GPU box with the tree).  Only tests load it, in a separate
process, because it has the same module name as this repo's own binding.

    python oracle/build_ref_binding.py <reference checkout root> [--force]
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT_DIR = os.path.join(HERE, "_ref")
LIB_DIR = os.path.join(REPO, "flash-attention-sm75-register-fused_b200", "lib")
MODULE = "flash_attn_sm75_cuda"


def out_path():
    return os.path.join(OUT_DIR, MODULE + sysconfig.get_config_var("EXT_SUFFIX"))


def build(ref_root, force=False, verbose=False):
    """Compile the reference binding into oracle/_ref/; returns the module
    path, or None when the reference checkout is absent."""
    src = os.path.join(ref_root, "src", "bindings", "pytorch_extension.cpp")
    if not os.path.exists(src):
        return None
    out = out_path()
    lib = os.path.join(LIB_DIR, "libfa_b200.so")
    if (not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src)
            and os.path.getmtime(out) >= os.path.getmtime(lib)):
        return out
    import torch
    from torch.utils import cpp_extension
    os.makedirs(OUT_DIR, exist_ok=True)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = cpp_extension.include_paths(device_type="cuda") + [
        sysconfig.get_paths()["include"], os.path.join(cuda_home, "include")]
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", src, "-o", out,
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={MODULE}",
           "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cmd += [f"-I{i}" for i in incs]
    cmd += [f"-L{d}" for d in libdirs] + [f"-L{LIB_DIR}", "-lfa_b200"]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
            f"-L{os.path.join(cuda_home, 'lib64')}", "-lcudart"]
    rel = os.path.relpath(LIB_DIR, OUT_DIR)
    cmd += [f"-Wl,-rpath,$ORIGIN/{rel}"] + [f"-Wl,-rpath,{d}" for d in libdirs]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("building the reference binding failed")
    return out


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: python oracle/build_ref_binding.py <reference checkout root> [--force]")
    print(build(sys.argv[1], force="--force" in sys.argv, verbose=True))
