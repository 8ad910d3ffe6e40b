import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden(name):
    import torch
    return torch.load(os.path.join(ROOT, "tests", "golden", name), weights_only=False)


@pytest.fixture(scope="session")
def cuda_lib():
    """The in-tree libpgf.so, loaded through the product's ctypes loader."""
    from icml_b200 import _lib
    return _lib.lib()
