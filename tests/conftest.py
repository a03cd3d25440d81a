import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def native_lib():
    """Builds (if stale) and loads libvauss_b200.so; fails loudly when missing."""
    from vauss_b200 import build, _native
    build.build()
    return _native.lib()


@pytest.fixture(scope="session")
def cuda(native_lib):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")
