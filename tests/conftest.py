import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def lib():
    from cngpt_b200 import abi
    return abi.load()


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device (no CPU fallback exists)"
    major, _ = torch.cuda.get_device_capability()
    assert major == 10, "libcngpt_cuda is built for sm_100a only"
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    return oracle
