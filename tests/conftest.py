"""Shared fixtures. Tests that need a B200 are marked ``gpu``; everything else runs on CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the built library")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def rb():
    """The product library on cuda:0, bound to torch's current stream. Fails (never skips) when
    the library or the GPU is missing, so a GPU run cannot pass on a fallback."""
    import torch
    import roaster_b200 as R
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.init()
    R.init(0)
    R.set_stream(torch.cuda.current_stream())
    return R
