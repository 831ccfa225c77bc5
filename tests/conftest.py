import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA C-ABI library)")
    config.addinivalue_line("markers", "slow: long-running oracle comparison")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def ref():
    from oracle import refcpu
    refcpu.lib()
    return refcpu


@pytest.fixture(autouse=True)
def _release_device_temporaries():
    yield
    if "tests.gpu_util" in sys.modules:
        try:
            sys.modules["tests.gpu_util"].release()
        except Exception:
            pass
