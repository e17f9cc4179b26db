import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    cap = torch.cuda.get_device_capability()
    if cap[0] < 10:
        pytest.fail(f"sm_100a kernels need a Blackwell GPU, found sm_{cap[0]}{cap[1]}")
    return torch.device("cuda:0")
