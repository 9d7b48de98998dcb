"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on CPU."""
import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def kats():
    with open(os.path.join(ROOT, "tests", "golden", "reference_kats.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def built_lib():
    """The in-tree libauratensor_cuda.so (rebuilt when a source is newer)."""
    from auratensor_b200 import build
    build.build()
    from auratensor_b200 import _lib
    return _lib.lib()


@pytest.fixture(scope="session")
def cuda(built_lib):
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")
