"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (they run on a B200 box); every other
test runs on the CPU.  The native libraries are (re)built in-tree before the
session when their sources changed; nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    from crumpet_b200 import _build

    _build.build()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
