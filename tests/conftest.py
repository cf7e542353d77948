"""Shared test setup: the `gpu` marker, repo root on sys.path, and common fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libmsattn.so")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request: pytest.FixtureRequest):
    """After every GPU test: no kernel may have left a status bit set (a bounded wait that gave
    up, an out-of-range slot, block or position).  Tests that plant such a fault read and clear
    the word themselves."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from miniserve_b200 import _capi

    status = _capi.device_status(int(torch.cuda.current_stream().cuda_stream))
    assert status == 0, f"a kernel left device status bits {status:#x} set during this test"
