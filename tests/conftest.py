"""Shared pytest setup: import paths, the ``gpu`` marker, golden fixtures."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
for path in (REPO, REPO / "pic-kvcache_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="session")
def store_sequence():
    return json.loads((GOLDEN / "store_sequence.json").read_text())


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
