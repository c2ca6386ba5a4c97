"""Shared test setup: the `gpu` marker, import paths for the package and the CPU oracle."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built libmira_cuda.so")


@pytest.fixture(scope="session")
def cuda_device():
    """Selects device 0 through the C ABI; fails (does not skip) when no GPU is usable, so a GPU
    run can never pass on a silent fallback."""
    from mira_b200 import _lib
    from mira_b200.device import set_device
    assert _lib.device_count() > 0, "no CUDA device visible to libmira_cuda.so"
    set_device(0)
    return 0
