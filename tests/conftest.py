"""Shared pytest configuration: the `gpu` marker, repo on sys.path, golden fixtures."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN_DIR / "reference_golden.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def cache_trace():
    return json.loads((GOLDEN_DIR / "cache_trace.json").read_text())


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test run without a CUDA device (deselect with -m 'not gpu')")
    from inferd_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)
