"""Shared test configuration.

Tests marked ``gpu`` need a B200 (sm_100a) and the built library; everything
else runs on the CPU.  GPU tests fail loudly without a GPU rather than skip:
a parity suite that skips proves nothing.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and libtorobi_b200.so")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def cuda():
    import torch

    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    import torobi_b200  # noqa: F401  (loads the library; raises if it is missing)

    torobi_b200.lib()
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.lib()
    return O


@pytest.fixture
def rng():
    import numpy as np

    return np.random.default_rng(int(os.environ.get("TQ_TEST_SEED", "1")))
