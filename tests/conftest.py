import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def kc_lib():
    from kudacuda_b200 import native

    return native.load_library()


@pytest.fixture(scope="session")
def kc_handle(kc_lib):
    import torch

    torch.cuda.init()
    handle = kc_lib.kudacuda_create(0)
    assert handle, "kudacuda_create returned null"
    assert kc_lib.kudacuda_freeze(handle) == 0, kc_lib.kudacuda_last_error(handle)
    yield handle
    torch.cuda.synchronize()
    kc_lib.kudacuda_destroy(handle)


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle

    oracle.build()
    return oracle
