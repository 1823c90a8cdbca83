"""Row-sharded FFN block (shard.RowShardedFfn) on one GPU with the ranks emulated in one process:
every rank's rows of gate / up / down, its SwiGLU slice quantized to Q8_K, and the all-gathers
replaced by concatenating the ranks' send buffers.  The reassembled output must equal the
unsharded FFN entry point (kq_run_ffn_async) and, for a few tokens, the oracle, bit for bit -- at
2, 4 and 8 ranks (uneven intermediate shares at 4 and 8)."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import shard, synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu

HIDDEN, FFN = 2560, 9728


@pytest.fixture(scope="module")
def ffn_weights():
    return (synth.gen_weights(kq.TYPE_Q4_K, FFN, HIDDEN, 301), synth.gen_weights(kq.TYPE_Q4_K, FFN, HIDDEN, 302),
            synth.gen_weights(kq.TYPE_Q6_K, HIDDEN, FFN, 303))


@pytest.mark.parametrize("M", [3, 64])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_sharded_ffn_emulated_ranks(kqctx, oracle, ffn_weights, world, M):
    import torch
    stream = torch.cuda.Stream()
    with kq.Context(0) as ctx, torch.cuda.stream(stream):
        ctx.set_stream(stream.cuda_stream)  # the library calls and the torch copies share one stream
        run_emulated(ctx, oracle, ffn_weights, world, M)
    torch.cuda.synchronize()


def run_emulated(kqctx, oracle, ffn_weights, world, M):
    import torch
    wg, wu, wd = ffn_weights
    x16 = synth.gen_activations(M, HIDDEN, 304 + M)
    gamma = (synth.gen_gamma(HIDDEN, 305).astype(np.float32) * 0.1).astype(np.float16)
    x = torch.from_numpy(x16.view(np.uint16).copy()).cuda().view(torch.float16).view(M, HIDDEN)
    gm = torch.from_numpy(gamma.view(np.uint16).copy()).cuda()
    full = [kqctx.upload(wg, kq.TYPE_Q4_K, FFN, HIDDEN), kqctx.upload(wu, kq.TYPE_Q4_K, FFN, HIDDEN),
            kqctx.upload(wd, kq.TYPE_Q6_K, HIDDEN, FFN)]
    y_ref = torch.zeros((M, HIDDEN), dtype=torch.float16, device="cuda")
    kqctx.run_ffn_async(*full, M, x, gm, y_ref)
    kqctx.synchronize()
    for W in full:
        W.free()
    plan = shard.FfnShardPlan(HIDDEN, FFN, world)
    ranks, weights, tasks = [], [], []
    for r in range(world):
        c0, C = plan.inter(r)
        r0, R = plan.hid(r)
        ws = (kqctx.upload(wg[c0:c0 + C], kq.TYPE_Q4_K, C, HIDDEN), kqctx.upload(wu[c0:c0 + C], kq.TYPE_Q4_K, C, HIDDEN),
              kqctx.upload(wd[r0:r0 + R], kq.TYPE_Q6_K, R, FFN))
        rk = shard.RowShardedFfn(kqctx, plan, r, M, "cuda")
        ranks.append(rk)
        weights.append(ws)
        tasks.append(rk.tasks(*ws, x))
    try:
        for rk, (gu, _) in zip(ranks, tasks):
            rk.part1(x, gm, gu)
        h_all = torch.cat([rk.h_send for rk in ranks])
        for rk, (_, dn) in zip(ranks, tasks):
            rk.h_all.copy_(h_all)
            rk.assemble_inter()
            rk.part2(dn)
        o_all = torch.cat([rk.o_send.view(-1) for rk in ranks])
        ys = []
        for rk in ranks:
            rk.o_all.copy_(o_all)
            y = torch.zeros((M, HIDDEN), dtype=torch.float16, device="cuda")
            rk.assemble_out(y)
            ys.append(y)
        kqctx.synchronize()
        want = bits(y_ref.cpu().numpy())
        for y in ys:
            assert np.array_equal(bits(y.cpu().numpy()), want)
        if M <= 4:
            ref = oracle.ffn(wg, kq.TYPE_Q4_K, wu, kq.TYPE_Q4_K, wd, kq.TYPE_Q6_K, HIDDEN, FFN, x16, gamma)
            assert np.array_equal(want, bits(ref))
    finally:
        for ws in weights:
            for W in ws:
                W.free()
