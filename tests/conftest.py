"""Shared pytest setup: import paths, the gpu marker, golden fixtures."""

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "helix-online-kv_b200")
for p in (PKG_ROOT, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(REPO, "tests", "golden", "reference_golden.npz")) as z:
        return {k: z[k] for k in z.files}
