"""Vocabulary-sharded LM head on two CPU ranks (torch.distributed gloo): every rank computes the
logits of its slice with the oracle, reduces it to per-row (value, row) pairs and the pairs are
all-gathered and merged.  The result must equal the single-process scan of the whole vocabulary
(the reference's first-maximal-row rule), including a tie planted across the slice boundary."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from npu880_mtk_npu_llm_runtime_b200 import shard, synth


def test_vocab_slices_cover_exactly():
    for vocab in (1, 7, 151936):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.vocab_slice(r, world, vocab) for r in range(world)]
            covered = []
            for first, n in spans:
                covered.extend(range(first, first + n))
            assert covered == list(range(vocab))


def test_merge_argmax_rules():
    vals = np.array([[1.0, 5.0, -np.inf], [3.0, 5.0, 2.0]], np.float32)
    rows = np.array([[10, 20, -1], [30, 7, 40]], np.int64)
    r, v = shard.merge_argmax(vals, rows)
    assert r.tolist() == [30, 7, 40] and v.tolist() == [3.0, 5.0, 2.0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V, K, M = 200, 256, 3
        w = synth.gen_weights(synth.TYPE_Q6_K, V, K, seed=61)
        x = synth.gen_activations(M, K, seed=62)
        O = Oracle()
        act = O.quantize_q8k(x)
        first, n = shard.vocab_slice(rank, world, V)
        logits = O.gemm(synth.TYPE_Q6_K, w[first:first + n], K, act)  # [M, n] fp32
        if rank == 1:
            logits[0, 0] = 1e9  # a tie with rank 0 below: the smaller global row must win
        if rank == 0:
            logits[0, n - 1] = 1e9
        i = logits.argmax(axis=1)  # first maximal row of the slice
        vals = torch.from_numpy(logits[np.arange(M), i].astype(np.float32))
        rows = torch.from_numpy((i + first).astype(np.int64))
        r, v = shard.gather_argmax_torch(vals, rows)
        q.put((rank, r.tolist(), v.tolist()))
    finally:
        dist.destroy_process_group()


def test_sharded_lm_head_gloo():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = [q.get(timeout=10) for _ in range(world)]
    # the single-process scan of the whole vocabulary with the same planted values
    from oracle.oracle import Oracle
    V, K, M = 200, 256, 3
    w = synth.gen_weights(synth.TYPE_Q6_K, V, K, seed=61)
    O = Oracle()
    act = O.quantize_q8k(synth.gen_activations(M, K, seed=62))
    full = O.gemm(synth.TYPE_Q6_K, w, K, act)
    half = shard.vocab_slice(1, world, V)[0]
    full[0, half] = 1e9
    full[0, half - 1] = 1e9
    ref_rows = full.argmax(axis=1).tolist()
    ref_vals = full[np.arange(M), full.argmax(axis=1)].tolist()
    for _, r, v in got:
        assert r == ref_rows and np.allclose(v, ref_vals, rtol=0, atol=0)


def _planted_logits(V, K, M):
    """the whole vocabulary's fp32 logits (oracle) with ties planted across slice boundaries for
    4 ranks: activation row 0 has its maximum at rows 1 and 2 (ranks 0 and 1), row 1 at rows 3 and
    4 (ranks 1 and 2)"""
    from oracle.oracle import Oracle
    w = synth.gen_weights(synth.TYPE_Q6_K, V, K, seed=63)
    O = Oracle()
    full = O.gemm(synth.TYPE_Q6_K, w, K, O.quantize_q8k(synth.gen_activations(M, K, seed=64)))
    full[0, 1] = full[0, 2] = 1e9
    full[1, 3] = full[1, 4] = 1e9
    return full


def _rank_main4(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V, K, M = 5, 256, 3
        first, n = shard.vocab_slice(rank, world, V)
        if n == 0:  # an empty slice contributes (-inf, row -1) for every activation row
            vals = torch.full((M,), float("-inf"))
            rows = torch.full((M,), -1, dtype=torch.int64)
        else:
            logits = _planted_logits(V, K, M)[:, first:first + n]
            i = logits.argmax(axis=1)
            vals = torch.from_numpy(logits[np.arange(M), i].astype(np.float32))
            rows = torch.from_numpy((i + first).astype(np.int64))
        r, v = shard.gather_argmax_torch(vals, rows)
        q.put((rank, n, r.tolist(), v.tolist()))
    finally:
        dist.destroy_process_group()


def test_sharded_lm_head_gloo_4_ranks_empty_slice():
    """4 ranks over a 5-row vocabulary (slices of 2, 2, 1 and 0 rows): ties across two slice
    boundaries go to the smaller row and the empty slice never wins"""
    import torch.multiprocessing as mp
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main4, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = [q.get(timeout=10) for _ in range(world)]
    assert sorted(n for _, n, _, _ in got) == [0, 1, 2, 2]
    full = _planted_logits(5, 256, 3)
    ref_rows = full.argmax(axis=1).tolist()
    assert ref_rows[:2] == [1, 3]
    ref_vals = full[np.arange(3), full.argmax(axis=1)].tolist()
    for _, _, r, v in got:
        assert r == ref_rows and v == ref_vals


# ---------------------------------------------------------------------------- FFN row sharding

FFN_HIDDEN, FFN_DIM, FFN_M = 512, 1280, 3  # 5 intermediate blocks: uneven shares at 2 and 4 ranks


def _ffn_inputs():
    wg = synth.gen_weights(synth.TYPE_Q4_K, FFN_DIM, FFN_HIDDEN, seed=71)
    wu = synth.gen_weights(synth.TYPE_Q4_K, FFN_DIM, FFN_HIDDEN, seed=72)
    wd = synth.gen_weights(synth.TYPE_Q6_K, FFN_HIDDEN, FFN_DIM, seed=73)
    x = synth.gen_activations(FFN_M, FFN_HIDDEN, seed=74)
    gamma = (synth.gen_gamma(FFN_HIDDEN, 75).astype(np.float32) * 0.1).astype(np.float16)
    return wg, wu, wd, x, gamma


def _ffn_rank_main(rank, world, port, q):
    """One rank of the row-sharded FFN block with the oracle for the products: its gate/up rows,
    SwiGLU and Q8_K of its intermediate slice, an all-gather of the Q8_K blocks, its rows of down
    with the residual, an all-gather of the output slices."""
    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle, Q8K_DTYPE
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        O = Oracle()
        wg, wu, wd, x, gamma = _ffn_inputs()
        plan = shard.FfnShardPlan(FFN_HIDDEN, FFN_DIM, world)
        M = FFN_M
        _, xq = O.rmsnorm(x, gamma)                                   # every rank: the whole row
        c0, C = plan.inter(rank)
        g = O.epilogue_f16(O.gemm(synth.TYPE_Q4_K, wg[c0:c0 + C], FFN_HIDDEN, xq))
        u = O.epilogue_f16(O.gemm(synth.TYPE_Q4_K, wu[c0:c0 + C], FFN_HIDDEN, xq))
        _, hq = O.swiglu(g, u)                                         # Q8_K of this slice
        pad = np.zeros((M, plan.inter_max), Q8K_DTYPE)
        pad[:, :C // 256] = hq
        got = torch.zeros((world * M, plan.inter_max * 292), dtype=torch.uint8)
        dist.all_gather_into_tensor(got, torch.from_numpy(pad.view(np.uint8).reshape(M, -1).copy()))
        blocks = got.view(world, M, plan.inter_max, 292).permute(1, 0, 2, 3).reshape(M, -1, 292)
        h_full = np.ascontiguousarray(blocks[:, torch.from_numpy(plan.inter_index())].numpy()).view(Q8K_DTYPE)
        h_full = h_full.reshape(M, FFN_DIM // 256)
        r0, R = plan.hid(rank)
        part = O.epilogue_f16(O.gemm(synth.TYPE_Q6_K, wd[r0:r0 + R], FFN_DIM, h_full),
                              np.ascontiguousarray(x[:, r0:r0 + R]))
        opad = np.zeros((M, plan.hid_max), np.float16)
        opad[:, :R] = part
        go = torch.zeros((world * M, plan.hid_max * 2), dtype=torch.uint8)  # fp16 bytes
        dist.all_gather_into_tensor(go, torch.from_numpy(opad.view(np.uint8).copy()))
        cols = go.view(world, M, plan.hid_max, 2).permute(1, 0, 2, 3).reshape(M, -1, 2)
        out = np.ascontiguousarray(cols[:, torch.from_numpy(plan.hid_index())].numpy())
        q.put((rank, C, R, out.tobytes()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_row_sharded_ffn_gloo(world):
    """The FFN block row-sharded over 2 / 4 CPU ranks (uneven intermediate shares, padded
    all-gathers) reassembles the single-process oracle result bit for bit on every rank."""
    import torch.multiprocessing as mp
    from oracle.oracle import Oracle
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ffn_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    got = [q.get(timeout=10) for _ in range(world)]
    wg, wu, wd, x, gamma = _ffn_inputs()
    ref = Oracle().ffn(wg, synth.TYPE_Q4_K, wu, synth.TYPE_Q4_K, wd, synth.TYPE_Q6_K, FFN_HIDDEN, FFN_DIM, x, gamma)
    plan = shard.FfnShardPlan(FFN_HIDDEN, FFN_DIM, world)
    assert sorted(c for _, c, _, _ in got) == sorted(plan.inter(r)[1] for r in range(world))
    assert len({c for _, c, _, _ in got}) == 2  # the shares really are uneven
    for _, _, _, b in got:
        assert b == ref.view(np.uint16).tobytes()
