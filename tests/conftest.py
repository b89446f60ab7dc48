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
def attention_golden():
    return np.load(GOLDEN / "attention.npz")


def element_values(bits: np.ndarray, dtype_code: int) -> np.ndarray:
    """uint16 bit patterns of bf16 (code 0) or fp16 (code 1) as fp32 values."""
    if dtype_code == 0:
        return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


@pytest.fixture(scope="session")
def store_sequence():
    return json.loads((GOLDEN / "store_sequence.json").read_text())


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
