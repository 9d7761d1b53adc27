"""Shared pytest configuration: the ``gpu`` marker and common fixtures."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (sm_100a) GPU and build/libqvelox.so')


@pytest.fixture(scope='session')
def lib():
    """The product library; a missing build is an error, never a skip."""
    from redshift_b200 import load_library
    return load_library()


@pytest.fixture(scope='session')
def hot():
    """Device-resident calls on torch CUDA tensors (GPU tests only)."""
    import torch
    assert torch.cuda.is_available(), 'GPU tests need a CUDA device'
    from redshift_b200 import HotPath
    return HotPath()
