"""Test configuration: registers the `gpu` marker and puts the product package
(minimax-h3-2xt4_b200/h3tp) and the repository root (oracle/) on sys.path."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "minimax-h3-2xt4_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libh3b200.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"sm_100 device required, found sm_{major}{minor}")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    return o
