import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")


def golden(name):
    return np.load(os.path.join(HERE, "golden", name))


@pytest.fixture
def device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return torch.device("cuda", 0)
