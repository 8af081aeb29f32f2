"""Test configuration: the `gpu` marker and shared fixtures.

Tests marked `gpu` need a CUDA device (a B200) and call the engine through
its C ABI; everything else runs on the CPU (the oracle against the golden
fixtures, the host-side logic, the library's exported symbols, and the
Scheme-A control plane over gloo).
"""

from __future__ import annotations

import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test is marked gpu and needs a CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
