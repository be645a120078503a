"""Shared test setup: import paths, the `gpu` marker and common fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (REPO / "orin-cuda-operator-library_b200", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture
def stream(cuda):
    """A non-default stream, as the reference's tests use
    (python/test_extension.py:30-51, tests/*.cu)."""
    import torch

    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        yield s
    s.synchronize()


@pytest.fixture(scope="session")
def ops(cuda):
    import operatorlib

    operatorlib.load_operatorlib()
    import torch

    return torch.ops.operatorlib
