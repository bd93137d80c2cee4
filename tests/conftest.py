import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def kats():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "reference_kats.npz"))


@pytest.fixture(scope="session")
def ane():
    """libane_b200 on a CUDA device (GPU tests only)."""
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import ane_b200

    return ane_b200
