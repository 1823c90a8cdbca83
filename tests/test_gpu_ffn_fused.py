"""The FFN block for 1-2 tokens as one persistent kernel (kq_ffn_fused.cu): bit for bit the
four-launch form and the oracle's restatement of the reference's FFN sequence (ENG:8283-8298)."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu


def _block(kqctx, oracle, gt, dt, hidden, ffn, M, seed, outlier=False):
    wg = synth.gen_weights(gt, ffn, hidden, seed)
    wu = synth.gen_weights(gt, ffn, hidden, seed + 1)
    wd = synth.gen_weights(dt, hidden, ffn, seed + 2)
    x = synth.gen_activations(M, hidden, seed + 3)
    if outlier:  # one large channel: the running sum of squares jumps several binades at once
        x[:, hidden // 3] = np.float16(180.0)
    gamma = (synth.gen_gamma(hidden, seed + 4).astype(np.float32) * 0.1).astype(np.float16)
    W = (kqctx.upload(wg, gt, ffn, hidden), kqctx.upload(wu, gt, ffn, hidden), kqctx.upload(wd, dt, hidden, ffn))
    return (wg, wu, wd), W, x, gamma


def _same(a, b):
    assert np.array_equal(np.isnan(a), np.isnan(b))
    ok = ~np.isnan(b)
    mism = int((bits(a)[ok] != bits(b)[ok]).sum())
    assert mism == 0, f"{mism} of {ok.sum()} fp16 outputs differ"


@pytest.mark.parametrize("gt,dt,hidden,ffn", [(kq.TYPE_Q4_K, kq.TYPE_Q6_K, 2560, 9728),
                                              (kq.TYPE_Q5_K, kq.TYPE_Q4_K, 1024, 2816),
                                              (kq.TYPE_Q4_K, kq.TYPE_Q5_K, 2048, 5632)])
@pytest.mark.parametrize("M", [1, 2])
def test_ffn_fused_equals_launches_and_oracle(kqctx, oracle, gt, dt, hidden, ffn, M):
    raw, W, x, gamma = _block(kqctx, oracle, gt, dt, hidden, ffn, M, 700 + 10 * M + hidden % 7,
                              outlier=(M == 2))
    try:
        fused = kqctx.run_ffn(*W, x, gamma)
        kqctx.set_option("ffn_fused", 0)
        try:
            launches = kqctx.run_ffn(*W, x, gamma)
        finally:
            kqctx.set_option("ffn_fused", 1)
    finally:
        for w in W:
            w.free()
    ref = oracle.ffn(raw[0], gt, raw[1], gt, raw[2], dt, hidden, ffn, x, gamma)
    _same(launches, ref)
    _same(fused, ref)


def test_ffn_fused_back_to_back(kqctx, oracle):
    """Several fused launches in a row on one stream (the grid barrier's words are reused by each
    launch): every output equals its own oracle result"""
    import torch
    hidden, ffn, M, n = 2560, 9728, 1, 6
    raw, W, _, gamma = _block(kqctx, oracle, kq.TYPE_Q4_K, kq.TYPE_Q6_K, hidden, ffn, M, 900)
    xs = [synth.gen_activations(M, hidden, 910 + i) for i in range(n)]
    try:
        gm = to_dev(gamma.view(np.uint16))
        xd = [to_dev(x.view(np.uint16)).view(torch.float16).view(M, hidden) for x in xs]
        yd = [torch.zeros((M, hidden), dtype=torch.float16, device="cuda") for _ in range(n)]
        for i in range(n):
            kqctx.run_ffn_async(*W, M, xd[i], gm, yd[i])
        kqctx.synchronize()
        outs = [y.cpu().numpy() for y in yd]
    finally:
        for w in W:
            w.free()
    for i in range(n):
        ref = oracle.ffn(raw[0], kq.TYPE_Q4_K, raw[1], kq.TYPE_Q4_K, raw[2], kq.TYPE_Q6_K, hidden, ffn, xs[i], gamma)
        _same(outs[i], ref)
