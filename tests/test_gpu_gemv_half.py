"""GEMV launches whose CTAs own 8-row halves of row groups (option "gemv_half", Q4_K / Q5_K, 1-2
activation rows): bit for bit the oracle and the whole-row-group form, on the shapes the plan
serves in halves -- the config-0 shape, a last row group with 8 rows, an odd number of 256-value
units per row, several tasks with unaligned row ranges -- and through the block-sum, fp16 +
residual and in-kernel-quantized input paths."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu


def _both(ctx, fn):
    """fn() with halves allowed (the default), then with whole row groups only"""
    a = fn()
    ctx.set_option("gemv_half", 0)
    try:
        b = fn()
    finally:
        ctx.set_option("gemv_half", 1)
    return a, b


# (type, K, [(weight rows, row_begin, rows)] per task)
SHAPES = [
    (kq.TYPE_Q4_K, 2560, [(9728, 0, 9728)]),               # config 0: 1,216 halves over 148 CTAs
    (kq.TYPE_Q4_K, 2560, [(10024, 0, 10024)]),             # last row group: 8 of 16 rows
    (kq.TYPE_Q5_K, 2560, [(8024, 0, 8024)]),
    (kq.TYPE_Q4_K, 1280, [(19024, 0, 19024)]),             # 5 units per row: an odd boundary pass
    (kq.TYPE_Q4_K, 512, [(17024, 0, 17024)]),
    (kq.TYPE_Q4_K, 2560, [(4100, 3, 4000), (4100, 0, 4100), (1700, 21, 1600)]),  # tasks, unaligned rows
]


@pytest.mark.parametrize("gtype,K,tasks", SHAPES, ids=["cfg0", "rows8", "q5k", "k1280", "k512", "tasks"])
def test_half_rows_bitexact(kqctx, oracle, gtype, K, tasks):
    import torch
    M = 1
    ws = [synth.gen_weights(gtype, n, K, seed=500 + 7 * i + n % 97) for i, (n, _, _) in enumerate(tasks)]
    Ws = [kqctx.upload(w, gtype, n, K) for w, (n, _, _) in zip(ws, tasks)]
    x = synth.gen_activations(M, K, seed=K + 11)
    act = oracle.quantize_q8k(x)
    try:
        def run():
            outs = [torch.full((M, r), float("nan"), dtype=torch.float32, device="cuda") for _, _, r in tasks]
            kqctx.gemm_multi_q8_async(to_dev(act), None, M, K,
                                      [dict(w=W, row_begin=b, rows=r, dst_f32=o)
                                       for W, (_, b, r), o in zip(Ws, tasks, outs)])
            kqctx.synchronize()
            return [o.cpu().numpy() for o in outs]
        got, whole = _both(kqctx, run)
    finally:
        for W in Ws:
            W.free()
    for w, (_, b, r), g, h in zip(ws, tasks, got, whole):
        ref = oracle.gemm(gtype, w[b:b + r], K, act)
        assert np.array_equal(bits(g), bits(ref)), f"max |diff| {np.abs(g - ref).max()}"
        assert np.array_equal(bits(h), bits(ref))


def test_half_rows_fp16_input_two_steps(kqctx, oracle):
    """fp16 input quantized in the kernel, two launches in a row"""
    import torch
    N, K = 9728, 2560
    w = synth.gen_weights(kq.TYPE_Q4_K, N, K, seed=77)
    W = kqctx.upload(w, kq.TYPE_Q4_K, N, K)
    try:
        for step in range(2):
            x = synth.gen_activations(1, K, seed=78 + step)
            xd = to_dev(x.view(np.uint16))
            out = torch.full((1, N), float("nan"), dtype=torch.float32, device="cuda")
            kqctx.gemm_multi_async(xd, 1, K, kqctx.make_tasks([dict(w=W, dst_f32=out, dst_f32_stride=N)]))
            kqctx.synchronize()
            ref = oracle.gemm(kq.TYPE_Q4_K, w, K, oracle.quantize_q8k(x))
            assert np.array_equal(bits(out.cpu().numpy()), bits(ref)), step
    finally:
        W.free()


def test_half_rows_block_sums(kqctx, oracle):
    """the per-block integer sums of a halves launch equal the reference's locals"""
    import torch
    rows, K, M = 9728, 2560, 1
    w = synth.gen_weights(kq.TYPE_Q4_K, rows, K, seed=81)
    x = synth.gen_activations(M, K, seed=82)
    act = oracle.quantize_q8k(x)
    W = kqctx.upload(w, kq.TYPE_Q4_K, rows, K)
    nb = K // 256
    try:
        si = torch.zeros((M, rows, nb), dtype=torch.int32, device="cuda")
        sm = torch.zeros_like(si)
        out = torch.zeros((M, rows), dtype=torch.float32, device="cuda")
        kqctx.debug_block_sums_async(W, 0, rows, to_dev(act), M, si, sm, out)
        kqctx.synchronize()
    finally:
        W.free()
    si, sm, out = si.cpu().numpy(), sm.cpu().numpy(), out.cpu().numpy()
    for r in list(range(0, 40)) + list(range(rows // 2 - 24, rows // 2 + 24)) + list(range(rows - 40, rows)):
        v, rsi, rsm = oracle.vec_dot(kq.TYPE_Q4_K, w[r], act[0], K)
        assert np.array_equal(si[0, r], rsi), r
        assert np.array_equal(sm[0, r], rsm), r
        assert bits(out[0, r]) == bits(v), r
    ref = oracle.gemm(kq.TYPE_Q4_K, w, K, act)
    assert np.array_equal(bits(out), bits(ref))


def test_half_rows_fp16_residual_dispatch(kqctx, oracle):
    """the dispatch epilogue (fp16 of sum + fp16 residual) from a halves launch"""
    N, K = 9728, 2560
    w = synth.gen_weights(kq.TYPE_Q4_K, N, K, seed=91)
    x = synth.gen_activations(1, K, seed=92)
    res = synth.gen_activations(1, N, seed=93)
    W = kqctx.upload(w, kq.TYPE_Q4_K, N, K)
    try:
        def run():
            d = np.zeros((1, N), np.float16)
            f = np.zeros((1, N), np.float32)
            kqctx.sdot_gemm_multi_dispatch(x, [dict(w=W, dst=d, residual=res, dst_f32=f)])
            return d, f
        (d, f), (d0, f0) = _both(kqctx, run)
    finally:
        W.free()
    ref = oracle.gemm(kq.TYPE_Q4_K, w, K, oracle.quantize_q8k(x))
    assert np.array_equal(bits(f), bits(ref))
    assert np.array_equal(bits(d), bits(oracle.epilogue_f16(ref, res)))
    assert np.array_equal(bits(d), bits(d0)) and np.array_equal(bits(f), bits(f0))
