"""In-tree build of the B200 attention library, its pybind module and CLIs.

Outputs (all next to the sources, so they travel with the tree):
  lib/libfa_b200.so                      C ABI (include/fa_b200.h), sm_100a kernels
  flash_attn_sm75_cuda<ext-suffix>.so    pybind module (reference's L3 name)
  lib/flash_mha_flatargs, lib/flash_mha_v2   standalone CLIs (reference argv/stdout)
  lib/libfa_selftest.so                  stage tests of the kernel's building blocks
                                         (loaded by tests/ only)

Every CUDA file is compiled with
  -gencode arch=compute_100a,code=sm_100a -lineinfo
nvcc cross-compiles, so this runs on a machine without a GPU.

    python build.py [--force] [-v]
"""
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
INC = os.path.join(REPO, "include")
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

KERNEL_SOURCES = ["fa_fwd_sm100.cu", "fa_abi.cu"]
KERNEL_HEADERS = ["sm100_ptx.cuh", "fa_softmax.cuh", "fa_fwd.h", "fa_bwd_sm100.cuh",
                  "fa_decode_sm100.cuh", "fa_fwd_tile.cuh", "fa_fwd_pair2.cuh"]


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=not verbose, text=True)
    if r.returncode != 0:
        if not verbose:
            sys.stderr.write(r.stdout or "")
            sys.stderr.write(r.stderr or "")
        raise RuntimeError(f"build step failed ({r.returncode}): {cmd[0]} ... {cmd[-1]}")
    return r


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def lib_path():
    return os.path.join(LIB, "libfa_b200.so")


def ext_path():
    return os.path.join(HERE, "flash_attn_sm75_cuda" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_lib(force=False, verbose=False):
    os.makedirs(LIB, exist_ok=True)
    out = lib_path()
    srcs = [os.path.join(CSRC, s) for s in KERNEL_SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in KERNEL_HEADERS] + [os.path.join(INC, "fa_b200.h")]
    if not force and not _stale(out, deps):
        return out
    objs = []
    for s in srcs:
        o = os.path.join(LIB, os.path.basename(s) + ".o")
        _run([NVCC, "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC",
              "-I", INC, "-I", CSRC, "-c", s, "-o", o], verbose)
        objs.append(o)
    _run([NVCC, "-shared", *ARCH, "-o", out, *objs, "-lcudart"], verbose)
    for o in objs:
        os.remove(o)
    return out


def build_ext(force=False, verbose=False):
    import torch
    from torch.utils import cpp_extension

    out = ext_path()
    src = os.path.join(CSRC, "pytorch_extension.cpp")
    if not force and not _stale(out, [src, lib_path(), os.path.join(INC, "fa_b200.h")]):
        return out
    incs = cpp_extension.include_paths(device_type="cuda") + [
        sysconfig.get_paths()["include"], INC, os.path.join(CUDA_HOME, "include")]
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC", src, "-o", out,
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=flash_attn_sm75_cuda",
           "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cmd += [f"-I{i}" for i in incs]
    cmd += [f"-L{d}" for d in libdirs] + [f"-L{LIB}", "-lfa_b200"]
    cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
            f"-L{os.path.join(CUDA_HOME, 'lib64')}", "-lcudart"]
    cmd += ["-Wl,-rpath,$ORIGIN/lib"] + [f"-Wl,-rpath,{d}" for d in libdirs]
    _run(cmd, verbose)
    return out


def build_cli(force=False, verbose=False):
    outs = []
    for name in ("flash_mha_flatargs", "flash_mha_v2"):
        src = os.path.join(CSRC, "cli", name + ".cu")
        common = os.path.join(CSRC, "cli", "cli_common.h")
        out = os.path.join(LIB, name)
        if not os.path.exists(src):
            continue
        if force or _stale(out, [src, common, lib_path()]):
            _run([NVCC, "-O3", "-std=c++17", *ARCH, "-lineinfo", "-I", INC, src, "-o", out,
                  f"-L{LIB}", "-lfa_b200", "-Xlinker", "-rpath,$ORIGIN"], verbose)
        outs.append(out)
    return outs


def selftest_path():
    return os.path.join(LIB, "libfa_selftest.so")


def build_selftest(force=False, verbose=False):
    """Test library of the kernel's building blocks (csrc/fa_selftest.cu):
    exp2 polynomial, softmax stage and single-tile tcgen05 products."""
    os.makedirs(LIB, exist_ok=True)
    out = selftest_path()
    src = os.path.join(CSRC, "fa_selftest.cu")
    deps = [src] + [os.path.join(CSRC, h) for h in ("sm100_ptx.cuh", "fa_softmax.cuh")]
    if force or _stale(out, deps):
        _run([NVCC, "-O3", "-std=c++17", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "-I", CSRC, src, "-o", out, "-lcudart"], verbose)
    return out


def build(force=False, verbose=False):
    build_lib(force, verbose)
    build_ext(force, verbose)
    build_cli(force, verbose)
    build_selftest(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built:", lib_path(), ext_path())
