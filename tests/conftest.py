"""Shared test set-up: repo root on sys.path, the `gpu` marker, and helpers.

`-m "not gpu"` runs the oracle against the reference's golden vectors, the
host logic and the ABI checks on the CPU; `-m gpu` runs the parity tests
through libdcfold.so's C ABI on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")
if GOLDEN_DIR not in sys.path:
    sys.path.insert(0, GOLDEN_DIR)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def dcf():
    """The product library on a GPU; the test fails loudly if it is missing."""
    import mlirpass_b200 as m
    assert os.path.exists(m.LIB_PATH), "libdcfold.so not built"
    assert have_gpu(), "gpu test without a GPU"
    m.init(1)
    return m
