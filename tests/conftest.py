"""Shared test setup: import paths and the `gpu` marker.

Tests marked `gpu` need a CUDA device and the built libsnn_b200.so; the rest
run on CPU (oracle against golden fixtures, host logic, C-ABI exports)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("pure-snn-language_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def root():
    return ROOT
