"""Row-group tile edge cases of the CUDA GEMV, bit-exact against the oracle.

The device layout groups weight rows by 16 (kq_common.cuh), the launch splits row groups over
the CTAs, and every (row, token) result is folded from its block terms in block order.  These
cases cover what the layout and the split make special: more row groups than SMs (several row
groups per CTA, a ring that wraps), task rows that start and end inside a row group, several
tasks of one type in one launch, the fp16 / residual epilogue on those rows, and a row count
that leaves the last row group partly padding."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu

TYPES = [kq.TYPE_Q4_K, kq.TYPE_Q5_K, kq.TYPE_Q6_K, kq.TYPE_Q8_0]


def q8_inputs(ctx, gtype, act):
    a = to_dev(act)
    return (None, a) if gtype == kq.TYPE_Q8_0 else (a, None)


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_many_row_groups(kqctx, oracle, gtype, M):
    """2603 rows = 163 row groups (> 148 SMs), the last one partly padding"""
    import torch
    rows, K = 2603, 512
    w = synth.gen_weights(gtype, rows, K, seed=500 + 7 * gtype + M)
    x = synth.gen_activations(M, K, seed=600 + M)
    act = oracle.act_for(gtype, x)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
        q8k, q80 = q8_inputs(kqctx, gtype, act)
        kqctx.gemm_multi_q8_async(q8k, q80, M, K, [dict(w=W, dst_f32=out)])
        kqctx.synchronize()
        got = out.cpu().numpy()
    finally:
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [1, 3])
def test_unaligned_tasks(kqctx, oracle, gtype, M):
    """three tasks of one type in one launch, rows starting and ending inside row groups, fp32
    and fp16 outputs, a residual on one of them"""
    import torch
    K = 768
    specs = [(90, 5, 37), (64, 16, 48), (40, 23, 17)]  # (weight rows, row_begin, rows)
    x = synth.gen_activations(M, K, seed=700 + M)
    act = oracle.act_for(gtype, x)
    ws, Ws, tasks, outs, outs16 = [], [], [], [], []
    res = torch.from_numpy(synth.gen_activations(M, 48, seed=701).view(np.uint16).copy()).to("cuda")
    try:
        for i, (wr, rb, n) in enumerate(specs):
            w = synth.gen_weights(gtype, wr, K, seed=800 + 10 * gtype + i)
            ws.append(w)
            Ws.append(kqctx.upload(w, gtype, wr, K))
            o = torch.full((M, n), float("nan"), dtype=torch.float32, device="cuda")
            o16 = torch.zeros((M, n), dtype=torch.float16, device="cuda")
            outs.append(o)
            outs16.append(o16)
            t = dict(w=Ws[-1], row_begin=rb, rows=n, dst_f32=o, dst=o16)
            if i == 1:
                t["residual"] = res
            tasks.append(t)
        q8k, q80 = q8_inputs(kqctx, gtype, act)
        kqctx.gemm_multi_q8_async(q8k, q80, M, K, tasks)
        kqctx.synchronize()
        for i, (wr, rb, n) in enumerate(specs):
            ref = oracle.gemm(gtype, ws[i][rb:rb + n], K, act)
            got = outs[i].cpu().numpy()
            assert np.array_equal(bits(got), bits(ref)), f"task {i}: max |diff| {np.abs(got - ref).max()}"
            ref16 = ref + (res.cpu().numpy().view(np.float16).astype(np.float32) if i == 1 else 0.0)
            ref16 = ref16.astype(np.float16)
            got16 = outs16[i].cpu().numpy()
            assert np.array_equal(got16.view(np.uint16), ref16.view(np.uint16)), f"task {i} fp16"
    finally:
        for W in Ws:
            W.free()


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
def test_dequant_tiled(kqctx, oracle, gtype):
    """dequantization reads the tiled layout back in GGUF order, rows inside row groups"""
    rows, K = 45, 512
    w = synth.gen_weights(gtype, rows, K, seed=900 + gtype)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        got = kqctx.dequant_rows(W, 7, 30)
    finally:
        W.free()
    ref = oracle.dequant(gtype, w[7:37], K)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
def test_embed_rows(kqctx, oracle, gtype):
    """embedding lookup: rows by token id (repeats, the last row, unsorted), host and device
    entry points, bit-exact to the reference's dequant of those rows; an id past the end is an
    error before anything runs (host) or a zero row and KQ_ERR_SHAPE at the next synchronize
    (device)"""
    import torch
    rows, K = 45, 768
    w = synth.gen_weights(gtype, rows, K, seed=950 + gtype)
    W = kqctx.upload(w, gtype, rows, K)
    ids = np.array([44, 3, 3, 17, 0, 31], np.uint32)
    try:
        got = kqctx.embed_rows(W, ids)
        ref = oracle.dequant(gtype, w[ids], K)
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
        with pytest.raises(kq.KQError) as e:
            kqctx.embed_rows(W, np.array([2, 45], np.uint32))
        assert e.value.status == -3
        dids = torch.from_numpy(np.array([5, 45, 7], np.uint32).view(np.int32)).cuda()
        out = torch.full((3, K), 1.0, dtype=torch.float16, device="cuda")
        kqctx.embed_rows_async(W, dids, 3, out)
        with pytest.raises(kq.KQError) as e:
            kqctx.synchronize()
        assert e.value.status == -3
        o = out.cpu().numpy()
        assert np.array_equal(o[0].view(np.uint16), oracle.dequant(gtype, w[5:6], K)[0].view(np.uint16))
        assert not o[1].any()
        assert np.array_equal(o[2].view(np.uint16), oracle.dequant(gtype, w[7:8], K)[0].view(np.uint16))
    finally:
        W.free()
