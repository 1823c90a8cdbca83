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


def rmsnorm_cases():
    """(M, K, x fp16, gamma fp16) RMSNorm cases: the benchmark hidden size at 1-64 rows, short and
    long rows (40,960 values: longer than the kernel stages squares for), small and large
    magnitudes, a zero row (sum 0), +-65504 and fp16 subnormals"""
    rng = np.random.default_rng(77)
    cases = []
    for M, K, scale in [(1, 2560, 1.0), (8, 2560, 1.0), (64, 2560, 1.0), (5, 256, 30.0), (3, 9728, 1.0),
                        (2, 2560, 1e-3), (2, 2560, 3000.0), (1, 40960, 1.0)]:
        x = (rng.standard_normal((M, K)) * scale).astype(np.float16)
        g = (rng.standard_normal(K) * 0.5 + 1.0).astype(np.float16)
        cases.append((M, K, x, g))
    x = np.zeros((3, 2560), np.float16)
    x[1, ::7] = np.float16(65504.0)
    x[1, 3::7] = np.float16(-65504.0)
    x[2] = (rng.standard_normal(2560) * 6e-5).astype(np.float16)
    cases.append((3, 2560, x, np.ones(2560, np.float16)))
    # rows whose running sum crosses binades in unusual ways: one outlier (several binades in one
    # add), magnitudes growing along the row, mostly zeros, a step pattern
    K = 2560
    i = np.arange(K)
    x = np.empty((4, K), np.float16)
    x[0] = (rng.standard_normal(K) * 0.1).astype(np.float16)
    x[0, K // 3] = np.float16(300.0)
    x[1] = (rng.standard_normal(K) * (1.0 + i / 100.0)).astype(np.float16)
    x[2] = np.where(i % 7 == 0, rng.standard_normal(K), 0.0).astype(np.float16)
    x[3] = np.where(i % 64 == 0, 8.0, 0.01).astype(np.float16)
    cases.append((4, K, x, (rng.standard_normal(K) * 0.5 + 1.0).astype(np.float16)))
    for M, K in [(2, 4096), (1, 65536)]:
        x = rng.standard_normal((M, K)).astype(np.float16)
        cases.append((M, K, x, (rng.standard_normal(K) * 0.5 + 1.0).astype(np.float16)))
    return cases


def all_fp16_gate(rows: int) -> np.ndarray:
    """every fp16 bit pattern once, as `rows` rows"""
    return np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16).reshape(rows, 65536 // rows)
