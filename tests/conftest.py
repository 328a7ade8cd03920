"""Shared test setup.

Markers:
  gpu   needs an sm_100 GPU (B200); everything else runs on CPU.

The product package lives in vllm-qdq-plugin_b200/ (directory name is not a
Python identifier), so it is put on sys.path here, as bench.py and
__graft_entry__.py do.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "vllm-qdq-plugin_b200"))
sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def golden(name: str):
    return np.load(GOLDEN / name)


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    if not gpu_available():
        pytest.skip("needs an sm_100 GPU")
    import torch
    return torch.device("cuda", 0)
