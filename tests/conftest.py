"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle against the golden fixtures, the host logic and
the C-ABI load/export checks; `-m gpu` runs the parity tests through the C-ABI
on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "flashrt-llama.cpp_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device; parity tests through the C-ABI")


@pytest.fixture(scope="session")
def O():
    from oracle import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def fr():
    import frb200
    frb200.lib()
    return frb200


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability(0)
    if major < 10:
        pytest.skip("needs an sm_100 device")
    return torch.device("cuda:0")
