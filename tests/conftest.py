"""Shared pytest configuration: the `gpu` marker and fixture loaders.

`-m "not gpu"` tests run on CPU (oracle vs golden fixtures, host logic, the
C-ABI surface); `-m gpu` tests need an sm_100 GPU and call the library.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")


@pytest.fixture(scope="session")
def mxfp8_golden():
    return np.load(GOLDEN / "mxfp8_golden.npz")


@pytest.fixture(scope="session")
def vda_golden():
    return np.load(GOLDEN / "vda_golden.npz")


@pytest.fixture(scope="session")
def vda_stages_golden():
    return np.load(GOLDEN / "vda_stages_golden.npz")


@pytest.fixture(scope="session")
def alpha_golden():
    return np.load(GOLDEN / "alpha_golden.npz")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for -m gpu tests")
    return torch.device("cuda", 0)
