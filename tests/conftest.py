import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "rdna-gfx1201-v0.1_b200")
for p in (REPO, PKG, os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests; fails (never skips) without a GPU."""
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    import q4rdna

    assert q4rdna.lib is not None, "libq4rdna.so must be built for gpu tests"
    return torch.device("cuda:0")
