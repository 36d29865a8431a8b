import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running test")
    config.addinivalue_line("markers", "distributed: spawns several processes")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from zeroq_b200.ops import _ext

    _ext.ext()  # fail loudly if the native extension is missing on a GPU machine
    return torch.device("cuda", 0)
