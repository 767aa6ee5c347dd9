"""Test configuration: import paths, the ``gpu`` marker, shared helpers.

``-m "not gpu"`` runs on a CPU-only host: the oracle against the golden
vectors, host-side logic, and the C ABI library's exports.  ``-m gpu`` runs
the parity tests that call the sm_100a kernels through the C ABI.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "mlx-flash_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; calls the sm_100a kernels")


@pytest.fixture(scope="session")
def golden():
    """Lazy loader for the committed golden fixtures."""
    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = np.load(os.path.join(GOLDEN, name), allow_pickle=False)
        return cache[name]

    return load


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("GPU test selected but no CUDA device is visible")
    return torch.device("cuda:0")
