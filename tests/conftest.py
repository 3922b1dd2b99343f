"""Pytest configuration: the `gpu` marker and repo-root imports.

Tests marked ``gpu`` need a CUDA device and the built library; everything
else runs on CPU (oracle checks, C-ABI exports, host-side logic, gloo ranks).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libtinygnn_b200.so")


def pytest_sessionstart(session):
    """A fresh checkout has no built library: build it (nvcc, sm_100a), the
    Python module over it and the oracle before any test needs them (the C++
    API test links the library without importing the package)."""
    from tinygnn_b200 import build
    build.ensure_built(pymodule=True)
    import oracle  # noqa: F401  (builds the C restatement when it is missing)


@pytest.fixture(scope="session")
def golden():
    from tests.helpers import load_golden
    return load_golden()


@pytest.fixture(scope="session")
def known_answers():
    from tests.helpers import load_known_answers
    return load_known_answers()
