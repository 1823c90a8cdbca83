"""Generate the golden fixtures in tests/golden/ by running the REFERENCE engine itself.

The reference (src/v182_r22_breakthrough_engine.c) ships no test vectors, so these fixtures
are produced by its own code, compiled unmodified from its sources by oracle/Makefile into
oracle/_ref/libkqref.so.  Every output below comes from a reference function:

* quantize_row_fp16_to_q8_k / _q8_0            (ENG:925, ENG:1016)
* sdot_row_<type>_batch, eval_single_lm_row_dot (ENG:1951, 3109, 3234, 3368, 10986)
* dequant_block_<type>                          (ENG:598, 673, 758, 803)
* rmsnorm_fp16_rows_fast, swiglu_fp16_rows_fast (ENG:4264, ENG:4361)
* sdot_gemm_multi_dispatch on the reference pool (ENG:4188), incl. the FFN call sequence
  of ENG:8283-8298.

Inputs are the seeded synthetic blocks of npu880_mtk_npu_llm_runtime_b200.synth.
Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from npu880_mtk_npu_llm_runtime_b200 import synth  # noqa: E402
from oracle.oracle import Reference, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
TYPES = {"q4_k": TYPE_Q4_K, "q5_k": TYPE_Q5_K, "q6_k": TYPE_Q6_K, "q8_0": TYPE_Q8_0}


def edge_activations(M: int, K: int, seed: int) -> np.ndarray:
    """Seeded N(0,1) rows plus the quantizer's edge cases: an all-zero row (d = 0 path,
    ENG:947-952), a row with one all-zero 32-block inside, and a row spanning the fp16 range."""
    x = synth.gen_activations(M, K, seed).astype(np.float32)
    if M >= 2:
        x[1, :] = 0.0
    if M >= 3:
        x[2, 32:64] = 0.0
        x[2, 5] = 60000.0
        x[2, 6] = -60000.0
        x[2, 7] = 1e-7
    return x.astype(np.float16)


def main() -> None:
    R = Reference()
    R.init_pool()
    cases = {}

    # per-type row dots, quantizers and dequantizers
    for name, t in TYPES.items():
        for (rows, K, M, seed) in [(16, 512, 3, 11), (8, 2560, 4, 12)]:
            w = synth.gen_weights(t, rows, K, seed=1000 * t + seed)
            x = edge_activations(M, K, seed=seed)
            act = R.quantize_q8_0(x) if t == TYPE_Q8_0 else R.quantize_q8k(x)
            out = R.gemm(t, w, K, act)
            # eval_single_lm_row_dot (the scalar LM-head row dot) for the K-quant types
            lm = np.array([R.lm_row_dot(t, w, K, act, r, 0) for r in range(rows)], dtype=np.float32) \
                if t != TYPE_Q8_0 else np.zeros(0, np.float32)
            deq = R.dequant(t, w, K)
            cases[f"dot_{name}_{rows}x{K}_m{M}"] = dict(type=np.int32(t), K=np.int32(K), w=w, x=x,
                                                       act=act.view(np.uint8).reshape(M, -1),
                                                       out=out, lm_out=lm, dequant=deq)

    # every value a GGUF file can hold: Q6_K scales over all of int8 (the reference's Q6_K
    # quantizer maps each block's largest scale to -128) and Q8_0 quants including -128
    for name, t, kw in [("q6_k_full", TYPE_Q6_K, dict(q6_scales=(-128, 128))),
                        ("q8_0_full", TYPE_Q8_0, dict(q8_quants=(-128, 128)))]:
        rows, K, M, seed = 16, 768, 3, 13
        w = synth.gen_weights(t, rows, K, seed=1000 * t + seed, **kw)
        x = edge_activations(M, K, seed=seed)
        act = R.quantize_q8_0(x) if t == TYPE_Q8_0 else R.quantize_q8k(x)
        out = R.gemm(t, w, K, act)
        lm = np.array([R.lm_row_dot(t, w, K, act, r, 0) for r in range(rows)], dtype=np.float32) \
            if t != TYPE_Q8_0 else np.zeros(0, np.float32)
        deq = R.dequant(t, w, K)
        cases[f"dot_{name}_{rows}x{K}_m{M}"] = dict(type=np.int32(t), K=np.int32(K), w=w, x=x,
                                                   act=act.view(np.uint8).reshape(M, -1),
                                                   out=out, lm_out=lm, dequant=deq)

    # sdot_gemm_multi_dispatch: two tasks sharing one input, fp16 output, residual on task 0
    K, M = 512, 3
    x = synth.gen_activations(M, K, 21)
    w0 = synth.gen_weights(TYPE_Q4_K, 40, K, 22)
    w1 = synth.gen_weights(TYPE_Q6_K, 24, K, 23)
    res0 = synth.gen_activations(M, 40, 24)
    d0 = np.zeros((M, 40), np.float16)
    d1 = np.zeros((M, 24), np.float16)
    R.dispatch(x, [(TYPE_Q4_K, w0, d0, res0), (TYPE_Q6_K, w1, d1, None)])
    cases["dispatch_q4k_q6k"] = dict(K=np.int32(K), x=x, w0=w0, w1=w1, res0=res0, dst0=d0, dst1=d1)

    # Q8_0 dispatch (quantizes the input to Q8_0, ENG:4212-4216)
    w2 = synth.gen_weights(TYPE_Q8_0, 20, K, 25)
    d2 = np.zeros((M, 20), np.float16)
    R.dispatch(x, [(TYPE_Q8_0, w2, d2, None)])
    cases["dispatch_q8_0"] = dict(K=np.int32(K), x=x, w=w2, dst=d2)

    # producers
    x = edge_activations(3, 768, 31)
    gamma = synth.gen_gamma(768, 32)
    xn, q = R.rmsnorm(x, gamma)
    cases["rmsnorm"] = dict(x=x, gamma=gamma, out=xn, q8k=q.view(np.uint8).reshape(3, -1))
    g = synth.gen_activations(3, 512, 33) * np.float16(3)
    u = synth.gen_activations(3, 512, 34)
    h, q = R.swiglu(g, u)
    cases["swiglu"] = dict(gate=g, up=u, out=h, q8k=q.view(np.uint8).reshape(3, -1))

    # FFN sequence ENG:8283-8298 at a small shape: rmsnorm(+Q8_K) -> {gate, up} Q4_K ->
    # swiglu(+Q8_K) -> down Q6_K + residual
    hidden, ffn, M = 256, 512, 3
    x = synth.gen_activations(M, hidden, 41)
    gamma = synth.gen_gamma(hidden, 42)
    wg = synth.gen_weights(TYPE_Q4_K, ffn, hidden, 43)
    wu = synth.gen_weights(TYPE_Q4_K, ffn, hidden, 44)
    wd = synth.gen_weights(TYPE_Q6_K, hidden, ffn, 45)
    xn, _ = R.rmsnorm(x, gamma)
    gate = np.zeros((M, ffn), np.float16)
    up = np.zeros((M, ffn), np.float16)
    R.dispatch(xn, [(TYPE_Q4_K, wg, gate, None), (TYPE_Q4_K, wu, up, None)], prequantized=True)
    h, _ = R.swiglu(gate, up)
    y = np.zeros((M, hidden), np.float16)
    R.dispatch(h, [(TYPE_Q6_K, wd, y, x)], prequantized=True)
    cases["ffn"] = dict(hidden=np.int32(hidden), ffn=np.int32(ffn), x=x, gamma=gamma, wg=wg, wu=wu, wd=wd,
                        gate=gate, up=up, h=h, out=y)

    # LM-head slice: fp16 logits of a Q6_K head through the dispatch (ENG:9686-9697)
    V, K = 300, 256
    w = synth.gen_weights(TYPE_Q6_K, V, K, 51)
    x = synth.gen_activations(2, K, 52)
    logits = np.zeros((2, V), np.float16)
    R.dispatch(x, [(TYPE_Q6_K, w, logits, None)])
    cases["lm_head_q6k"] = dict(K=np.int32(K), w=w, x=x, logits=logits)

    for name, arrs in cases.items():
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **arrs)
    total = sum(os.path.getsize(os.path.join(OUT, f"{n}.npz")) for n in cases)
    print(f"wrote {len(cases)} fixtures, {total / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
