"""Parity of the tensor-core (tcgen05 int8 MMA) path used for M > 8 activation rows.

The per-(row, sub-block) scales are split into byte-sized pieces (one MMA each) and recombined
in int32, and the fp32 block terms are added in block order, so every result is compared
BIT-EXACTLY with the oracle: fp32 outputs, fp16 outputs with a residual, both input forms
(fp16 activation quantized in the library, or pre-quantized Q8_K / Q8_0 blocks), row ranges that
start and end inside row groups and token counts that leave the last token tile partly empty."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev
from test_gpu_split import check_q80_tolerance

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=[1, 3], ids=["rowmajor", "tokenmajor"])
def force_tensor_cores(kqctx, request):
    """pin a tensor-core kernel (the default chooses by a cost model): 1 = weight rows as the
    MMA's A operand, 3 = activation tokens as A in tensor memory"""
    kqctx.set_option("gemm_path", request.param)
    yield
    kqctx.set_option("gemm_path", 0)


TYPES = [kq.TYPE_Q4_K, kq.TYPE_Q5_K, kq.TYPE_Q6_K, kq.TYPE_Q8_0]


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M,rows,K", [(9, 130, 512), (64, 300, 2560), (100, 1030, 768)])
def test_tc_prequantized_bitexact(kqctx, oracle, gtype, M, rows, K):
    import torch
    w = synth.gen_weights(gtype, rows, K, seed=1100 + 3 * gtype + M)
    x = synth.gen_activations(M, K, seed=1200 + M)
    act = oracle.act_for(gtype, x)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
        a = to_dev(act)
        q8k, q80 = (None, a) if gtype == kq.TYPE_Q8_0 else (a, None)
        kqctx.gemm_multi_q8_async(q8k, q80, M, K, [dict(w=W, dst_f32=out)])
        kqctx.synchronize()
        got = out.cpu().numpy()
    finally:
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
def test_tc_fp16_input_tasks_residual(kqctx, oracle, gtype):
    """fp16 input quantized by the library, two tasks with unaligned row ranges, fp16 + fp32
    outputs, a residual on the second task"""
    import torch
    M, K = 70, 1024
    specs = [(200, 7, 150), (64, 16, 40)]
    x16 = synth.gen_activations(M, K, seed=1300)
    act = oracle.act_for(gtype, x16)
    ws, Ws, tasks, o32, o16 = [], [], [], [], []
    res = torch.from_numpy(synth.gen_activations(M, 40, seed=1301).view(np.uint16).copy()).to("cuda")
    try:
        for i, (wr, rb, n) in enumerate(specs):
            w = synth.gen_weights(gtype, wr, K, seed=1400 + 10 * gtype + i)
            ws.append(w)
            Ws.append(kqctx.upload(w, gtype, wr, K))
            a = torch.full((M, n), float("nan"), dtype=torch.float32, device="cuda")
            b = torch.zeros((M, n), dtype=torch.float16, device="cuda")
            o32.append(a)
            o16.append(b)
            t = dict(w=Ws[-1], row_begin=rb, rows=n, dst_f32=a, dst=b)
            if i == 1:
                t["residual"] = res
            tasks.append(t)
        xd = torch.from_numpy(x16.view(np.uint16).copy()).to("cuda")
        kqctx.gemm_multi_async(xd, M, K, tasks)
        kqctx.synchronize()
        for i, (wr, rb, n) in enumerate(specs):
            ref = oracle.gemm(gtype, ws[i][rb:rb + n], K, act)
            got = o32[i].cpu().numpy()
            assert np.array_equal(bits(got), bits(ref)), f"task {i}: max |diff| {np.abs(got - ref).max()}"
            r16 = ref + (res.cpu().numpy().view(np.float16).astype(np.float32) if i == 1 else 0.0)
            assert np.array_equal(o16[i].cpu().numpy().view(np.uint16), r16.astype(np.float16).view(np.uint16))
    finally:
        for W in Ws:
            W.free()


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [12, 32, 48, 64])
def test_tc_split_k(kqctx, oracle, gtype, M):
    """few rows and a long K: the row-major kernel splits K over CTAs, stores the block terms and
    a fold kernel adds them in unit order (fp32, fp16 + residual, an unaligned row range).  At
    M = 48 / 64 it runs two 32-token tiles with K split instead of one 64-token tile.  Q8_0's split
    terms are per-unit sums of its eight 32-block terms (check_q80_tolerance); the others bit-exact."""
    import torch
    rows_w, rb, n, K = 320, 5, 290, 4096
    w = synth.gen_weights(gtype, rows_w, K, seed=1700 + gtype + M)
    x = synth.gen_activations(M, K, seed=1701 + M)
    act = oracle.act_for(gtype, x)
    res = torch.from_numpy(synth.gen_activations(M, n, seed=1702).view(np.uint16).copy()).to("cuda")
    W = kqctx.upload(w, gtype, rows_w, K)
    try:
        o32 = torch.full((M, n), float("nan"), dtype=torch.float32, device="cuda")
        o16 = torch.zeros((M, n), dtype=torch.float16, device="cuda")
        a = to_dev(act)
        q8k, q80 = (None, a) if gtype == kq.TYPE_Q8_0 else (a, None)
        kqctx.gemm_multi_q8_async(q8k, q80, M, K, [dict(w=W, row_begin=rb, rows=n, dst_f32=o32, dst=o16, residual=res)])
        kqctx.synchronize()
        got = o32.cpu().numpy()
        got16 = o16.cpu().numpy()
    finally:
        W.free()
    ref = oracle.gemm(gtype, w[rb:rb + n], K, act)
    r16 = (ref + res.cpu().numpy().view(np.float16).astype(np.float32)).astype(np.float16)
    if gtype == kq.TYPE_Q8_0:
        check_q80_tolerance(got, ref, got16, r16)
        return
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"
    assert np.array_equal(got16.view(np.uint16), r16.view(np.uint16))


@pytest.mark.parametrize("gtype,M,rows", [(kq.TYPE_Q6_K, 16, 256), (kq.TYPE_Q6_K, 64, 2560), (kq.TYPE_Q8_0, 64, 2560)],
                         ids=["q6_k-16", "q6_k-64", "q8_0-64"])
def test_tc_ffn_down_shape(kqctx, oracle, gtype, M, rows):
    """the FFN down projection shape (K = 9728): Q6_K (tree verify) at M = 16 (256 rows) and at
    M = 64 (all 2,560 rows: 32-token tiles with K split), and Q8_0 (the batched-decode stack's
    down projection) at M = 64 with per-unit split terms (check_q80_tolerance)"""
    import torch
    K = 9728
    w = synth.gen_weights(gtype, rows, K, seed=1500)
    x = synth.gen_activations(M, K, seed=1501)
    act = oracle.act_for(gtype, x)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
        a = to_dev(act)
        kqctx.gemm_multi_q8_async(None if gtype == kq.TYPE_Q8_0 else a, a if gtype == kq.TYPE_Q8_0 else None, M, K,
                                  [dict(w=W, dst_f32=out)])
        kqctx.synchronize()
        got = out.cpu().numpy()
    finally:
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    if gtype == kq.TYPE_Q8_0:
        check_q80_tolerance(got, ref)
        return
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"


@pytest.mark.parametrize("path", [0, 2])
def test_other_paths_agree(kqctx, oracle, path):
    """the cost-model choice and the forced GEMV tiles give the same bits for M > 8"""
    import torch
    kqctx.set_option("gemm_path", path)
    gtype, M, rows, K = kq.TYPE_Q4_K, 20, 200, 2560
    w = synth.gen_weights(gtype, rows, K, seed=1600)
    x = synth.gen_activations(M, K, seed=1601)
    act = oracle.act_for(gtype, x)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
        kqctx.gemm_multi_q8_async(to_dev(act), None, M, K, [dict(w=W, dst_f32=out)])
        kqctx.synchronize()
        got = out.cpu().numpy()
    finally:
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref))
