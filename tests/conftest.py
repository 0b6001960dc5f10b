"""pytest configuration: the ``gpu`` marker and shared fixtures.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on CPU.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden.npz")))


@pytest.fixture(autouse=True)
def _release_device_buffers():
    yield
    mod = sys.modules.get("gpu_util")
    if mod is not None:
        mod.ALIVE.clear()
