"""pytest configuration: import paths and the `gpu` marker.

`-m "not gpu"` runs everything that needs no GPU (oracle vs golden fixtures,
host logic, C-ABI exports, multi-process gloo tests); `-m gpu` runs the CUDA
parity tests, which call the kernels through the C ABI.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "kernelbench-hip_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
