"""Shared pytest setup: the ``gpu`` marker and helpers to load the golden fixtures."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C-ABI")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"golden_{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session", params=["g1", "g2"])
def golden_graph(request):
    return request.param, load_golden(request.param)


@pytest.fixture(scope="session")
def golden_reducers():
    return load_golden("reducers")
