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
