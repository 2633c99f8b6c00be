"""Shared pytest setup.

Markers: `gpu` tests need a CUDA device and the built libhale_cuda.so; the
driver runs `-m "not gpu"` on a CPU-only machine and `-m gpu` on a B200.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libhale_cuda.so")


def hale_pkg():
    """The product package (its directory name has a dash, so import by name)."""
    return importlib.import_module("hale-token_b200")


@pytest.fixture(scope="session")
def hale():
    return hale_pkg()
