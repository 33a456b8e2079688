"""Shared pytest setup.

- Puts the repo root (for ``oracle``) and ``musa-aiter_b200/`` (for the
  ``musa_aiter`` package) on ``sys.path``.
- Registers the ``gpu`` marker: tests that need a CUDA device.  The CPU suite
  runs with ``-m "not gpu"``.
- Seeds torch for every test (the reference suite does the same,
  op_tests/conftest.py:15-30).
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "musa-aiter_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(autouse=True)
def _seed():
    import torch

    torch.manual_seed(42)
    yield


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
