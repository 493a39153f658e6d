import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


def pytest_collection_modifyitems(config, items):
    # tests/test_zz_* files are collected last by name; keep that order stable
    items.sort(key=lambda it: (os.path.basename(str(it.fspath)).startswith("test_zz"), ))


@pytest.fixture(scope="session")
def oracle():
    from tests import oracle_lib
    return oracle_lib.Oracle()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import q27_b200
    if q27_b200._lib.lib().q27_device_arch() != 1000:
        pytest.fail("the engine is built for sm_100a only and this device is not one")
    return torch.device("cuda:0")
