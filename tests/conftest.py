"""Shared pytest configuration for the trnfft_b200 test suite."""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built trnfft_b200 library")


@pytest.fixture(scope="session")
def golden():
    """Loader for the reference-generated fixtures in tests/golden/*.npz."""
    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
        return cache[name]

    return load


@pytest.fixture
def rng():
    """Seeded NumPy generator (the reference seeds torch with 42, tests/conftest.py:11-13)."""
    return np.random.default_rng(42)
