"""Shared pytest setup: the `gpu` marker, repository imports and fixture loaders."""
from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA kernels")


def golden_files(prefix: str = ""):
    return sorted(glob.glob(os.path.join(GOLDEN, f"{prefix}*.npz")))


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name if name.endswith(".npz") else name + ".npz")) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()
