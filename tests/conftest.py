import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


@pytest.fixture(autouse=True)
def _seed_torch():
    """Every test starts from the same torch generator state (CPU and CUDA), so data drawn
    without an explicit generator does not depend on which tests ran before."""
    import torch
    torch.manual_seed(20240)
