"""Shared fixtures. Tests marked `gpu` need a B200 (cuda:0) and call the
CUDA path through the C ABI; everything else runs on the CPU."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (cuda:0); calls the CUDA path")


@pytest.fixture(scope="session")
def ce():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def O():
    from oracle import oracle
    return oracle


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("this test needs a CUDA device (it is marked gpu)")
    torch.cuda.set_device(0)
    return torch.device("cuda:0")
