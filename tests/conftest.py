import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def felix():
    """The C ABI of libfelix_b200.so (built in-tree). Fails loudly if missing."""
    from sion_b200 import abi
    return abi


@pytest.fixture(autouse=True)
def _clean_watchdog(request):
    """Every GPU test must leave the device watchdog word clear."""
    yield
    if "gpu" in request.keywords and _has_gpu():
        from sion_b200 import abi
        code = abi.watchdog_status(clear=True)
        assert code == 0, f"device watchdog fired (site {code})"
