"""Pytest configuration: the `gpu` marker and seeded RNGs.

GPU tests (``@pytest.mark.gpu``) run the hand-written sm_100a kernels through
the C ABI and compare them with the CPU oracle in ``oracle/``; CPU tests pin
the oracle against the golden fixtures in ``tests/golden/`` and check the
host logic and the library's exported symbols.
"""

from __future__ import annotations

import random
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _seed_everything() -> None:
    """Seed Python, NumPy and PyTorch RNGs for reproducible tests."""
    random.seed(42)
    np.random.seed(42)
    torch.manual_seed(42)
