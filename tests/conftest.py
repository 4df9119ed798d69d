"""Shared fixtures (mirrors the reference's ``tests/conftest.py:7-17``)."""

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from skmetal_b200._config import PER_ESTIMATOR_THRESHOLDS, _set_thread_device, get_config  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libskmetal_cuda.so")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly (not skip) when the CUDA path is missing on a GPU
    # run; on a CPU-only machine they are skipped so `-m "not gpu"` stays clean.
    from skmetal_b200 import _bridge

    if _bridge.GPU_AVAILABLE:
        return
    have_gpu_env = os.environ.get("SKMETAL_REQUIRE_GPU") == "1"
    for item in items:
        if "gpu" in item.keywords and not have_gpu_env:
            item.add_marker(pytest.mark.skip(reason="no CUDA GPU visible"))


@pytest.fixture(autouse=True)
def reset_config():
    cfg = get_config()
    cfg.device = "gpu"
    _set_thread_device(None)
    cfg.threshold = 1
    cfg.dtype = "float32"
    cfg.verbose = False
    cfg.thresholds = dict(PER_ESTIMATOR_THRESHOLDS)
    cfg.gpu_index = 0
    yield
