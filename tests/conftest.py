"""Shared pytest configuration.

* ``gpu`` marks tests that need a CUDA device (an sm_100 B200); the CPU suite runs with
  ``-m "not gpu"``.
* Every test starts from ``torch.manual_seed(0)`` as the reference's suite does
  (prism_infer tests/conftest.py:48-51).
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")


@pytest.fixture(autouse=True)
def _seed():
    import torch
    torch.manual_seed(0)


@pytest.fixture
def expert_engine():
    """Select the library's expert GEMM engine for one test (``auto`` again afterwards)."""
    from prism_infer_b200 import capi
    yield capi.set_expert_engine
    capi.set_expert_engine("auto")


def load_golden(name):
    import numpy as np
    return dict(np.load(GOLDEN / f"{name}.npz", allow_pickle=False))
