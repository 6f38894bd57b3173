"""Shared pytest configuration.

Markers:
  gpu -- needs a CUDA device (a B200); everything else runs on the CPU.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(ROOT, "tests", "golden", "quantization_golden.npz"))


@pytest.fixture(scope="session")
def native_lib():
    """The product library, built in-tree if it is missing."""
    from zyron_b200 import build

    build.build()
    from zyron_b200 import _lib

    return _lib.lib()


@pytest.fixture(scope="session")
def cuda(native_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
