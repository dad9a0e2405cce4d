import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: runs CUDA kernels on a B200 (sm_100a) device")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for GPU tests; fails (never skips) when there is none,
    so a GPU run cannot pass on a silent fallback."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test requires a CUDA device")
    from hard_resets_compose_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)
