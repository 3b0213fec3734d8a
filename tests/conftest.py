import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "ns_golden.pt")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN)


@pytest.fixture(scope="session")
def cuda_lib():
    """The native library on a GPU box; the test fails loudly if it is absent."""
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device")
    from muon_fused import _lib

    return _lib.load()
