"""The vocabulary-sharded LM head with its all-gather inside the GEMV (kq_peer_gather): ranks
emulated on one GPU (every rank's gather is issued before any wait, on one stream, so no kernel
waits for one that has not run), checked bit for bit against one unsharded GEMV; and the bounded
wait when a rank never publishes."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import shard, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("M", [1, 3])
def test_peer_gather_emulated_ranks(kqctx, world, M):
    import torch
    V, K = 1000, 512
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, seed=60 + world)
    full = kqctx.upload(w, kq.TYPE_Q6_K, V, K)
    slices = []
    for r in range(world):
        r0, n = shard.vocab_slice(r, world, V)
        slices.append(kqctx.upload(w[r0:r0 + n], kq.TYPE_Q6_K, n, K))
    gs = shard.PeerGather.emulated(kqctx, world, M, V)
    try:
        for step in range(3):  # both buffers, then the first again
            x = torch.from_numpy(synth.gen_activations(M, K, 70 + step).view(np.uint16).copy()).cuda()
            ref = torch.zeros((M, V), dtype=torch.float32, device="cuda")
            kqctx.gemm_multi_async(x, M, K, kqctx.make_tasks([dict(w=full, dst_f32=ref, dst_f32_stride=V)]))
            for r in range(world):
                gs[r].gather(slices[r], x)
            outs = [torch.full((M, gs[0].row_stride), float("nan"), dtype=torch.float32, device="cuda")
                    for _ in range(world)]
            for r in range(world):
                gs[r].wait(outs[r])
            kqctx.synchronize()
            want = ref.cpu().numpy().view(np.uint32)
            for r in range(world):
                got = outs[r][:, :V].cpu().numpy().view(np.uint32)
                assert np.array_equal(got, want), (step, r)
    finally:
        for g in gs:
            g.close()
        for W in slices + [full]:
            W.free()


def test_peer_gather_wait_times_out(kqctx):
    """A rank that never publishes: the wait gives up after the context's timeout, the call reports
    KQ_ERR_TIMEOUT and the context keeps working."""
    import torch
    V, K, M = 512, 256, 1
    w = synth.gen_weights(kq.TYPE_Q4_K, V, K, seed=80)
    r0, n = shard.vocab_slice(0, 2, V)
    W0 = kqctx.upload(w[r0:r0 + n], kq.TYPE_Q4_K, n, K)
    gs = shard.PeerGather.emulated(kqctx, 2, M, V)
    x = torch.from_numpy(synth.gen_activations(M, K, 81).view(np.uint16).copy()).cuda()
    kqctx.set_option("timeout_ms", 20)
    try:
        gs[0].gather(W0, x)  # rank 1 never runs its slice
        gs[0].wait(None)
        with pytest.raises(kq.KQError) as ei:
            kqctx.synchronize()
        assert ei.value.status == -7  # KQ_ERR_TIMEOUT
    finally:
        kqctx.set_option("timeout_ms", 1000)
        for g in gs:
            g.close()
    out = torch.zeros((M, n), dtype=torch.float32, device="cuda")
    kqctx.gemm_multi_async(x, M, K, kqctx.make_tasks([dict(w=W0, dst_f32=out, dst_f32_stride=n)]))
    kqctx.synchronize()
    assert np.isfinite(out.cpu().numpy()).all()
    W0.free()


def test_peer_gather_in_kernel_completion_one_rank(kqctx):
    """The step completed inside the GEMV (out given, no wait call): with one rank the kernel's tail
    CTAs only count the step; over 3 steps (both buffers) out equals an unsharded GEMV, and a
    following gather + wait pair (the other form) sees the steps counted"""
    import torch
    V, K, M = 1000, 512, 2
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, seed=95)
    W = kqctx.upload(w, kq.TYPE_Q6_K, V, K)
    (g,) = shard.PeerGather.emulated(kqctx, 1, M, V)
    try:
        for step in range(4):
            x = torch.from_numpy(synth.gen_activations(M, K, 96 + step).view(np.uint16).copy()).cuda()
            ref = torch.zeros((M, V), dtype=torch.float32, device="cuda")
            kqctx.gemm_multi_async(x, M, K, kqctx.make_tasks([dict(w=W, dst_f32=ref, dst_f32_stride=V)]))
            out = torch.full((M, V), float("nan"), dtype=torch.float32, device="cuda")
            if step < 3:
                g.gather(W, x, out)
            else:
                g.gather(W, x)
                g.wait(out)
            kqctx.synchronize()
            assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32)), step
    finally:
        g.close()
        W.free()
