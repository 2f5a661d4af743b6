"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200) and the built extension;
everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "popkv_golden.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built popkv_b200 library")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN) as data:
        return {name: data[name] for name in data.files}


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
