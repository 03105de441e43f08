"""The C-ABI library loads, exports every function include/fa_b200.h declares,
and rejects bad arguments before touching a GPU (no compute calls here)."""
import ctypes

import pytest

from tests import abi_ctypes as abi


def test_library_exports_every_header_function():
    lib = ctypes.CDLL(abi.LIB_PATH)
    declared = abi.header_functions()
    assert len(declared) >= 14
    missing = [n for n in declared if not hasattr(lib, n)]
    assert missing == []
    # the ctypes signature table covers the whole header
    assert sorted(abi.SIGNATURES) == declared


def test_reference_launcher_names_are_exported():
    lib = ctypes.CDLL(abi.LIB_PATH)
    for name in ("launch_flash_attention_forward", "launch_flash_attention_forward_scalar",
                 "launch_flash_attention_forward_wmma_qk", "launch_naive_attention",
                 "flatargs_launch", "launch_v2"):
        assert hasattr(lib, name)


def test_argument_errors_before_launch():
    lib = abi.load()
    n = None
    # unsupported head_dim (the reference's error text)
    assert lib.fa_fwd(n, n, n, n, n, 1, 1, 1, 16, 96, 1.0, 0, 0, n) == 2
    assert b"head_dim=64 or 128" in lib.fa_error_string(2)
    assert lib.fa_fwd(n, n, n, n, n, 1, 1, 1, 16, 64, 1.0, 0, 7, n) == 5      # dtype
    assert lib.fa_fwd(n, n, n, n, n, 1, 1, 1, 16, 64, 1.0, 2, 0, n) == 1      # causal flag
    assert lib.fa_fwd(n, n, n, n, n, -1, 1, 1, 16, 64, 1.0, 0, 0, n) == 1     # negative size
    assert lib.fa_fwd(n, n, n, n, n, 1, 6, 4, 16, 64, 1.0, 0, 0, n) == 3      # GQA divisibility
    assert lib.fa_fwd(n, n, n, n, n, 1, 4, 0, 16, 64, 1.0, 0, 0, n) == 1      # Hkv == 0
    assert lib.fa_fwd(n, n, n, n, n, 1, 4, 2, 16, 64, 1.0, 0, 0, n) == 1      # null pointers
    p = ctypes.c_void_p(0x1003)  # misaligned
    assert lib.fa_fwd(p, p, p, p, n, 1, 4, 2, 16, 64, 1.0, 0, 0, n) == 4
    # empty problems are no-ops (nothing launched)
    assert lib.fa_fwd(n, n, n, n, n, 0, 4, 2, 16, 64, 1.0, 0, 0, n) == 0
    assert lib.fa_fwd(n, n, n, n, n, 1, 4, 2, 0, 64, 1.0, 0, 0, n) == 0
    assert lib.launch_v2(n, n, n, n, 1, 1, 16, 1.0, 5, n) == 1               # bad mode


def test_diagnostics():
    lib = abi.load()
    assert lib.fa_version().startswith(b"fa_b200")
    assert 150 * 1024 < lib.fa_smem_bytes(64) <= 227 * 1024
    assert 150 * 1024 < lib.fa_smem_bytes(128) <= 227 * 1024
    assert lib.fa_smem_bytes(96) == -1
    for code in range(0, 11):
        assert lib.fa_error_string(code)
    assert b"watchdog" in lib.fa_error_string(110)


def test_header_is_plain_c():
    text = open(abi.HEADER).read()
    assert 'extern "C"' in text
    import re
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)  # declarations only, not comments
    for forbidden in ("torch", "at::", "Tensor", "std::"):
        assert forbidden not in text


def test_selftest_library_exports_its_stage_tests():
    """The test-only library of the kernel's building blocks (exp2 polynomial,
    softmax stage, single-tile tcgen05 products) loads without a GPU."""
    import os
    path = os.path.join(os.path.dirname(abi.LIB_PATH), "libfa_selftest.so")
    lib = ctypes.CDLL(path)
    for name in ("fa_selftest_exp2", "fa_selftest_softmax", "fa_selftest_mma"):
        assert hasattr(lib, name)
