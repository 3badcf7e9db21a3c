import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the snn_b200 library on it")


@pytest.fixture(scope="session")
def gpu_count():
    import torch
    return torch.cuda.device_count()
