"""The C restatement (oracle/kq_oracle.c) reproduces the reference engine's own outputs.

The golden fixtures were produced by running the unmodified reference engine
(tests/golden/make_golden.py).  Every comparison is bit-exact: integer/byte outputs by value,
fp32/fp16 outputs by bit pattern.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import golden_files, load_golden
from oracle.oracle import Q8K_DTYPE, Q8_0_DTYPE, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view({2: np.uint16, 4: np.uint32}[a.dtype.itemsize])


DOT_FILES = golden_files("dot_")


def test_fixtures_present():
    assert len(DOT_FILES) == 10, "golden fixtures missing: run tests/golden/make_golden.py"


@pytest.mark.parametrize("path", DOT_FILES, ids=[os.path.basename(p)[:-4] for p in DOT_FILES])
def test_quantize_and_row_dot(oracle, path):
    g = load_golden(path)
    t, K = int(g["type"]), int(g["K"])
    act = oracle.act_for(t, g["x"])
    # activation quantizer: d, qs, bsum32 byte-identical (ENG:925-990 / ENG:1016-1064)
    assert act.view(np.uint8).reshape(act.shape[0], -1).tobytes() == g["act"].tobytes()
    out = oracle.gemm(t, g["w"], K, act)
    assert np.array_equal(bits(out), bits(g["out"]))
    if t != TYPE_Q8_0:
        # eval_single_lm_row_dot for token 0 (ENG:10986)
        assert np.array_equal(bits(out[0]), bits(g["lm_out"]))
    deq = oracle.dequant(t, g["w"], K)
    assert np.array_equal(bits(deq), bits(g["dequant"]))


def test_quantizer_edge_cases(oracle):
    g = load_golden(DOT_FILES[0])
    act = oracle.act_for(int(g["type"]), g["x"])
    # all-zero row -> d = 0, zero quants and sums (ENG:947-952)
    assert np.all(act[1]["d"] == 0) and not act[1]["qs"].any() and not act[1]["bsum32"].any()
    # clamp to +-127 (ENG:980-981) on the row that spans the fp16 range
    assert act[2]["qs"].max() <= 127 and act[2]["qs"].min() >= -127


def test_dispatch_two_tasks(oracle):
    g = load_golden("dispatch_q4k_q6k")
    K = int(g["K"])
    act = oracle.quantize_q8k(g["x"])
    d0 = oracle.epilogue_f16(oracle.gemm(TYPE_Q4_K, g["w0"], K, act), g["res0"])
    d1 = oracle.epilogue_f16(oracle.gemm(TYPE_Q6_K, g["w1"], K, act))
    assert np.array_equal(bits(d0), bits(g["dst0"]))
    assert np.array_equal(bits(d1), bits(g["dst1"]))


def test_dispatch_q8_0(oracle):
    g = load_golden("dispatch_q8_0")
    K = int(g["K"])
    out = oracle.epilogue_f16(oracle.gemm(TYPE_Q8_0, g["w"], K, oracle.quantize_q8_0(g["x"])))
    assert np.array_equal(bits(out), bits(g["dst"]))


def test_rmsnorm_and_swiglu(oracle):
    g = load_golden("rmsnorm")
    out, q = oracle.rmsnorm(g["x"], g["gamma"])
    assert np.array_equal(bits(out), bits(g["out"]))
    assert q.view(np.uint8).reshape(q.shape[0], -1).tobytes() == g["q8k"].tobytes()
    g = load_golden("swiglu")
    h, q = oracle.swiglu(g["gate"], g["up"])
    assert np.array_equal(bits(h), bits(g["out"]))
    assert q.view(np.uint8).reshape(q.shape[0], -1).tobytes() == g["q8k"].tobytes()


def test_ffn_sequence(oracle):
    g = load_golden("ffn")
    hidden, ffn = int(g["hidden"]), int(g["ffn"])
    out = oracle.ffn(g["wg"], TYPE_Q4_K, g["wu"], TYPE_Q4_K, g["wd"], TYPE_Q6_K, hidden, ffn, g["x"], g["gamma"])
    assert np.array_equal(bits(out), bits(g["out"]))


def test_lm_head_logits_and_argmax(oracle):
    g = load_golden("lm_head_q6k")
    K = int(g["K"])
    act = oracle.quantize_q8k(g["x"])
    bi, bv, logits = oracle.rows_argmax(TYPE_Q6_K, g["w"], K, act, f16_compare=True, want_logits=True)
    f16 = oracle.epilogue_f16(logits)
    assert np.array_equal(bits(f16), bits(g["logits"]))
    ref_best = np.argmax(g["logits"].astype(np.float32), axis=1)   # first maximal index
    assert np.array_equal(bi.astype(np.int64), ref_best)


def test_row_bytes(oracle):
    # compute_ggml_bytes, ENG:364-374
    assert oracle.row_bytes(12, 2560) == 1440
    assert oracle.row_bytes(13, 2560) == 1760
    assert oracle.row_bytes(14, 2560) == 2100
    assert oracle.row_bytes(14, 9728) == 7980
    assert oracle.row_bytes(8, 2560) == 2720
    assert oracle.row_bytes(99, 2560) == 0


def test_q8k_layout():
    assert Q8K_DTYPE.itemsize == 292 and Q8_0_DTYPE.itemsize == 36
