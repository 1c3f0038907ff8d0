"""Shared pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle, host-logic and ABI-load tests on a CPU-only
machine; `-m gpu` runs the CUDA parity tests on a B200.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "beacon-ai_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_lib():
    """The C-ABI library, loaded once per session (GPU tests only)."""
    if not has_gpu():
        pytest.fail("GPU test collected on a machine without a CUDA device")
    from beacon_cuda import _lib
    return _lib.lib()
