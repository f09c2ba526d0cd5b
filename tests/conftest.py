"""Shared pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs everywhere (oracle vs reference goldens, C-ABI exports,
host-side logic, gloo multi-process logic); `-m gpu` needs a B200 and calls
the CUDA backend through its C ABI.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "iris.c_b200"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200) and the built libiris_cuda.so")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def iris():
    """The loaded libiris_cuda binding; GPU tests fail loudly if it is missing."""
    import iris_cuda
    iris_cuda.lib()
    assert iris_cuda.lib().iris_cuda_init(0) == 0, iris_cuda.last_error()
    return iris_cuda
