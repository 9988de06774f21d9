"""Shared test setup.

``-m "not gpu"`` runs on a CPU-only machine: oracle vs golden fixtures, host
logic, and loading of the C-ABI library.  ``-m gpu`` tests need a B200 and
compare the CUDA path with the oracle through the C ABI.
"""
import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 GPU (B200)")


def load_pkg():
    return importlib.import_module("mxfp8-grouped-gemm_b200")


@pytest.fixture(scope="session")
def mxg():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    from oracle import mxfp8_oracle
    return mxfp8_oracle


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    return torch.device("cuda", 0)
