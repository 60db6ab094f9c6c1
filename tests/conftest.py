"""Shared pytest configuration.

Markers: ``gpu`` -- needs a B200 and the built CUDA library (``pytest -m gpu``);
everything else runs on the CPU (``pytest -m "not gpu"``).
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "genie-tk_b200")
for p in (REPO, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
