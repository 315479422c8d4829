import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# Before CUDA starts: more hardware queues, so the emulated drives' copy streams
# rarely share one with a stream whose work waits on an io kernel.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")
# Eager kernel loading: a lazy load while an io kernel waits on the drives
# would stall the drives' copy calls (a context-wide lock) until its deadline.
os.environ.setdefault("CUDA_MODULE_LOADING", "EAGER")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "multigpu: needs 2+ CUDA devices")


def _cuda():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords or "multigpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture
def tmp_root(tmp_path):
    return tmp_path
