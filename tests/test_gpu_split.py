"""Balanced GEMV launches ("gemv_split"): where whole row groups would spread unevenly over the
SMs, CTAs own equal ranges of 16-row x 256-value tiles instead, so a row group can be shared by
two or many neighbouring CTAs; the last CTA to finish a shared row group adds its block terms in
block order.  Every case is bit-exact against the oracle, except Q8_0 rows too long for per-block
terms at this M (check_q80_tolerance).

Covered: row groups spread over dozens of CTAs (few rows, long K), all four weight types, 1..8
activation rows, fp16 input (quantized in the kernel) and pre-quantized input (staged with
cp.async), fp16 + residual epilogue, back-to-back launches (the arrival counts must return to
zero), the same launch with the split off, and a launch after one that stopped on a timeout."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu

TYPES = [kq.TYPE_Q4_K, kq.TYPE_Q5_K, kq.TYPE_Q6_K, kq.TYPE_Q8_0]


def check_q80_tolerance(got, ref, got16=None, ref16=None):
    """Q8_0 rows too long for one shared-memory term per 32-value block at this M are summed one
    term per 256-value tile: the same products, another fp32 summation order.  Tolerance: 1e-5
    of the output scale (fp32); that plus one fp16 ulp of the value (fp16 outputs)."""
    tol = 1e-5 * np.abs(ref).max()
    assert np.all(np.abs(got - ref) <= tol), f"max |diff| {np.abs(got - ref).max()}"
    if got16 is not None:
        g, r = got16.astype(np.float32), ref16.astype(np.float32)
        assert np.all(np.abs(g - r) <= tol + np.spacing(np.abs(ref16)).astype(np.float32))


def run(ctx, gtype, W, rows, K, x16, act, fp16_input, residual=None):
    import torch
    M = x16.shape[0]
    out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
    out16 = torch.zeros((M, rows), dtype=torch.float16, device="cuda")
    task = dict(w=W, dst_f32=out, dst=out16)
    if residual is not None:
        task["residual"] = residual
    if fp16_input:
        xd = torch.from_numpy(x16.view(np.uint16).copy()).cuda()
        ctx.gemm_multi_async(xd, M, K, [task])
    else:
        a = to_dev(act)
        ctx.gemm_multi_q8_async(None if gtype == kq.TYPE_Q8_0 else a, a if gtype == kq.TYPE_Q8_0 else None, M, K,
                                [task])
    ctx.synchronize()
    return out.cpu().numpy(), out16.cpu().numpy()


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [1, 2, 5, 8])
@pytest.mark.parametrize("fp16_input", [False, True], ids=["q8", "fp16"])
def test_row_groups_over_many_ctas(kqctx, oracle, gtype, M, fp16_input):
    """37 rows x K = 16384: 3 row groups of 64 tiles over up to 296 CTAs (each row group shared
    by dozens of CTAs; the last row group partly padding).  Q8_0 at K = 4096 (48 one-tile CTAs,
    16 per row group): its per-block term order (bit-exact) needs 8 terms per tile in shared
    memory, which longer rows at 8 tokens do not leave room for."""
    rows, K = 37, (4096 if gtype == kq.TYPE_Q8_0 else 16384)
    w = synth.gen_weights(gtype, rows, K, seed=1100 + 7 * gtype + M)
    x16 = synth.gen_activations(M, K, seed=1200 + M)
    act = oracle.act_for(gtype, x16)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        got, _ = run(kqctx, gtype, W, rows, K, x16, act, fp16_input)
    finally:
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_back_to_back_and_split_off(kqctx, oracle, gtype, M):
    """2560 x 9728 (the FFN down shape: 160 row groups of 38 tiles over 148 SMs): three launches
    in a row with different inputs, fp16 outputs with a residual, then the split switched off.
    Bit-exact, except Q8_0 beyond 2 tokens (check_q80_tolerance)."""
    import torch
    rows, K = 2560, 9728
    w = synth.gen_weights(gtype, rows, K, seed=1300 + gtype)
    W = kqctx.upload(w, gtype, rows, K)
    res = torch.from_numpy(synth.gen_activations(M, rows, seed=1301).view(np.uint16).copy()).cuda()
    res_np = res.cpu().numpy().view(np.float16).astype(np.float32)
    try:
        for it, split in enumerate([1, 1, 1, 0]):
            kqctx.set_option("gemv_split", split)
            x16 = synth.gen_activations(M, K, seed=1400 + 10 * M + it)
            act = oracle.act_for(gtype, x16)
            got, got16 = run(kqctx, gtype, W, rows, K, x16, act, fp16_input=(it % 2 == 1), residual=res)
            ref = oracle.gemm(gtype, w, K, act)
            ref16 = (ref + res_np).astype(np.float16)
            if gtype == kq.TYPE_Q8_0 and M > 2:
                check_q80_tolerance(got, ref, got16, ref16)
                continue
            assert np.array_equal(bits(got), bits(ref)), f"launch {it}: max |diff| {np.abs(got - ref).max()}"
            assert np.array_equal(got16.view(np.uint16), ref16.view(np.uint16)), f"launch {it}: fp16"
    finally:
        kqctx.set_option("gemv_split", 1)
        W.free()


def test_split_after_timeout(kqctx, oracle):
    """a launch that stops on a wait timeout may leave arrival counts behind; the next balanced
    launch on the context must still be exact"""
    gtype, rows, K, M = kq.TYPE_Q4_K, 300, 4096, 2
    w = synth.gen_weights(gtype, rows, K, seed=1500)
    W = kqctx.upload(w, gtype, rows, K)
    x16 = synth.gen_activations(M, K, seed=1501)
    act = oracle.act_for(gtype, x16)
    try:
        kqctx.set_option("timeout_ms", 20)
        kqctx.set_option("inject_timeout", 1)
        with pytest.raises(kq.KQError) as ei:
            run(kqctx, gtype, W, rows, K, x16, act, fp16_input=False)
        assert ei.value.status == -7  # KQ_ERR_TIMEOUT
        kqctx.set_option("inject_timeout", 0)
        got, _ = run(kqctx, gtype, W, rows, K, x16, act, fp16_input=False)
    finally:
        kqctx.set_option("inject_timeout", 0)
        kqctx.set_option("timeout_ms", 1000)
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref))
