"""Shared pytest set-up: the `gpu` marker and import paths.

CPU tests (``-m "not gpu"``) cover the oracle against the golden fixtures, the
host-side logic and the C-ABI library's exported symbols.  GPU tests
(``-m gpu``) are the parity tests proper; they need an sm_100 device and the
in-tree build (``python __graft_entry__.py`` or ``build.py``).
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "flash-attention-sm75-register-fused_b200")
for p in (REPO, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built extension")


def _has_sm100():
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0)[0] == 10
    except Exception:
        return False


HAS_SM100 = _has_sm100()


@pytest.fixture(scope="session")
def sm100():
    if not HAS_SM100:
        pytest.fail("GPU test selected but no sm_100 device is visible")
    return True
