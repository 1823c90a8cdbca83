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


@pytest.fixture(scope="session")
def kqctx():
    """A libkq context on cuda:0 (GPU tests only)."""
    import torch
    import npu880_mtk_npu_llm_runtime_b200 as kq
    from npu880_mtk_npu_llm_runtime_b200 import build as kqbuild
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    kqbuild.build()
    torch.cuda.init()
    ctx = kq.Context(0)
    yield ctx
    ctx.close()


def to_dev(a):
    """numpy array -> torch CUDA tensor with the same bytes (structured arrays as uint8)."""
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype.fields is not None or a.dtype == np.uint32:
        a = a.view(np.uint8)
    return torch.from_numpy(a.copy()).cuda()


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view({1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[a.dtype.itemsize])
