"""Test configuration: import paths, the ``gpu`` marker and shared helpers."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "depth-anything-v2_b200", ROOT / "oracle", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libdav2_b200.so")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def dav2lib():
    """The product library; on a GPU box its absence is a failure, not a skip."""
    import dav2_b200

    return dav2_b200.load()


@pytest.fixture(scope="session")
def cuda(dav2lib):
    if not cuda_available():
        pytest.fail("CUDA device required for gpu-marked tests")
    import torch

    torch.cuda.init()
    return torch


def max_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
