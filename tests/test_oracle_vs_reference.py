"""The C restatement (oracle/kq_oracle.c) against the reference engine itself, compiled from its
unmodified sources into oracle/_ref (oracle/Makefile), on seeded inputs beyond the committed
fixtures: every weight type, K from one super-block to the reference input buffer's 9216, 1 to 32
tokens (its M limit), full-range Q6_K scales and Q8_0 quants, all-zero activation blocks and
activations at the fp16 extremes.  Quantizer bytes, per-row fp32 products (sdot_row_<type>_batch),
eval_single_lm_row_dot and dequant are compared bit for bit.  Skipped where the reference was not
built (its sources are absent)."""
from __future__ import annotations

import numpy as np
import pytest

from npu880_mtk_npu_llm_runtime_b200 import synth
from oracle.oracle import TYPE_Q8_0, reference_available
from conftest import all_fp16_gate, rmsnorm_cases

TYPES = [synth.TYPE_Q4_K, synth.TYPE_Q5_K, synth.TYPE_Q6_K, synth.TYPE_Q8_0]

pytestmark = pytest.mark.skipif(not reference_available(), reason="reference engine not built (oracle/_ref)")


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import Reference
    return Reference()


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view({2: np.uint16, 4: np.uint32}[a.dtype.itemsize])


def activations(M, K, seed):
    """N(0,1) rows, then edge rows: an all-zero super-block, fp16 extremes (+-65504, subnormals)"""
    x = synth.gen_activations(M, K, seed)
    if M >= 2:
        x[1, :256] = 0
    if M >= 3:
        x[2, ::7] = np.float16(65504.0)
        x[2, 3::11] = np.float16(-65504.0)
        x[2, 5::13] = np.float16(6e-8)
    return x


def check(oracle, ref, gtype, rows, K, M, seed, **wopts):
    w = synth.gen_weights(gtype, rows, K, seed=seed, **wopts)
    x = activations(M, K, seed + 1)
    if gtype == TYPE_Q8_0:
        a_o, a_r = oracle.quantize_q8_0(x), ref.quantize_q8_0(x)
    else:
        a_o, a_r = oracle.quantize_q8k(x), ref.quantize_q8k(x)
    assert a_o.tobytes() == a_r.tobytes()
    out_o = oracle.gemm(gtype, w, K, a_o)
    out_r = ref.gemm(gtype, w, K, a_r)
    assert np.array_equal(bits(out_o), bits(out_r))
    if gtype != TYPE_Q8_0:
        for r, m in ((0, 0), (rows - 1, M - 1), (rows // 2, M // 2)):
            assert bits(np.float32(ref.lm_row_dot(gtype, w, K, a_r, r, m))) == bits(out_o[m, r])
    assert np.array_equal(bits(oracle.dequant(gtype, w, K)), bits(ref.dequant(gtype, w, K)))


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("K,M", [(256, 1), (2560, 5), (4096, 32), (9216, 3)])
def test_oracle_equals_reference(oracle, ref, gtype, K, M):
    check(oracle, ref, gtype, 24, K, M, seed=500 + 17 * gtype + K + M)


@pytest.mark.parametrize("gtype,opts", [(synth.TYPE_Q6_K, dict(q6_scales=(-128, 128))),
                                        (synth.TYPE_Q8_0, dict(q8_quants=(-128, 128)))],
                         ids=["q6_k_full_scales", "q8_0_full_quants"])
def test_oracle_equals_reference_full_range(oracle, ref, gtype, opts):
    check(oracle, ref, gtype, 40, 2560, 8, seed=900 + gtype, **opts)


def test_rmsnorm_oracle_equals_reference(oracle, ref):
    """rmsnorm_fp16_rows_fast (ENG:4264-4314): the oracle's sequential fp32 sum of squares and
    rounding steps give the compiled reference's fp16 rows (and Q8_K where the reference makes
    one: M <= 32, K <= 9216) on the cases the GPU test uses"""
    for M, K, x, gamma in rmsnorm_cases():
        o, oq = oracle.rmsnorm(x, gamma)
        r, rq = ref.rmsnorm(x, gamma)
        assert np.array_equal(bits(o), bits(r)), (M, K)
        if M <= 32 and K <= 9216:
            fin = np.isfinite(r).all(axis=1)
            assert oq[fin].tobytes() == rq[fin].tobytes()


@pytest.mark.parametrize("up_kind", ["ones", "random"])
def test_swiglu_oracle_equals_reference_all_fp16(oracle, ref, up_kind):
    """swiglu_fp16_rows_fast (ENG:4326-4383) over every fp16 gate value (32 rows x 2048, the
    reference's input buffer holds 32 rows): the oracle's libm expf path gives the compiled
    reference's fp16 outputs bit for bit (NaN where it is NaN) and its Q8_K of all-finite rows"""
    gate = all_fp16_gate(32)
    rng = np.random.default_rng(5)
    up = (np.ones(gate.shape, np.float16) if up_kind == "ones"
          else (rng.standard_normal(gate.shape) * 2.0).astype(np.float16))
    o, oq = oracle.swiglu(gate, up)
    r, rq = ref.swiglu(gate, up)
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(o), nan)
    assert np.array_equal(bits(o)[~nan], bits(r)[~nan])
    fin = np.isfinite(r).all(axis=1)
    assert oq[fin].tobytes() == rq[fin].tobytes()
