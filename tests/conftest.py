import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


@pytest.fixture(scope="session")
def oracle():
    from tests._oracle import Oracle
    return Oracle.load()


@pytest.fixture(scope="session")
def qrc():
    import quickruncuda_b200 as q
    return q


@pytest.fixture(scope="session")
def lib():
    from quickruncuda_b200 import _native
    return _native.load(False)


@pytest.fixture(scope="session")
def lib_checked():
    from quickruncuda_b200 import _native
    return _native.load(True)


@pytest.fixture(scope="session")
def cuda():
    """The GPU tests' device.  A missing GPU is a failure, not a skip: these
    tests only run where a B200 is expected."""
    import torch
    assert torch.cuda.is_available(), "GPU test collected on a machine without CUDA"
    major, _ = torch.cuda.get_device_capability(0)
    assert major == 10, f"expected an sm_100 device, got compute capability {major}.x"
    return torch.device("cuda:0")
