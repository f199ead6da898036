"""Shared test setup: import paths, the ``gpu`` marker, fixture loaders."""

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rvc-vulkan_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_meta():
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        return json.load(f)


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def pytest_collection_modifyitems(config, items):
    """A GPU run needs the CUDA library: when any selected test is marked
    ``gpu``, loading librvc_cuda.so is checked once up front, so a missing or
    broken build fails the run loudly instead of skipping its tests."""
    if any(it.get_closest_marker("gpu") for it in items):
        from rvc_cuda import _lib  # noqa: F401,PLC0415  (raises ImportError when the library is missing)
