import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


@pytest.fixture(autouse=True)
def seed():
    torch.manual_seed(0)


def has_gpu() -> bool:
    return torch.cuda.is_available()


requires_gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
