"""Shared pytest setup: import paths and the `gpu` marker.

Tests marked ``gpu`` need a CUDA device (run with ``-m gpu`` on a B200); the rest
run on CPU (``-m "not gpu"``).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "star-kv-serve_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
