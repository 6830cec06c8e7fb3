import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and libpacuda.so")


def _gpu_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _gpu_present():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this machine")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def ctx():
    """A libpacuda context on cuda:0. On a GPU machine a missing or unloadable library is an error, not a skip."""
    import backburner_b200 as pa
    if not pa.available():
        raise RuntimeError("libpacuda.so did not load on this GPU machine: " + pa.lib_path)
    c = pa.Context(0)
    yield c
    c.close()
