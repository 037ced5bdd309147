"""Shared pytest configuration.

Markers: ``gpu`` -- needs a CUDA device (B200, sm_100a); every other test runs on the
CPU.  The engine package directory name is not a Python identifier, so it is loaded
through ``__graft_entry__.load_package()`` as ``tko_b200``.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__ as g

    return g.load_package()


@pytest.fixture(scope="session")
def cuda(pkg):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    pkg.load_library()
    return torch.device("cuda:0")
