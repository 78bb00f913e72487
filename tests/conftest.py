import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) GPU")


def cuda_ok() -> bool:
    import torch

    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def ogx_lib():
    """The built C-ABI library (built in-tree on first use)."""
    from opengenie_b200 import _lib, build

    build.build()
    return _lib.load()
