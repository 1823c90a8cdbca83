"""Parity of the CUDA K-quant GEMV (through the C ABI) with the oracle and with the reference's
own golden outputs.  Integer block sums and fp32 results are compared BIT-EXACTLY: the kernels
add the per-block fp32 terms in block order with the reference's operation sequence."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, golden_files, load_golden, to_dev

pytestmark = pytest.mark.gpu

TYPES = [kq.TYPE_Q4_K, kq.TYPE_Q5_K, kq.TYPE_Q6_K, kq.TYPE_Q8_0]


def run_q8(ctx, W, gtype, act, M, K, rows, row_begin=0):
    import torch
    out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
    a = to_dev(act)
    if gtype == kq.TYPE_Q8_0:
        ctx.gemm_multi_q8_async(None, a, M, K, [dict(w=W, row_begin=row_begin, rows=rows, dst_f32=out)])
    else:
        ctx.gemm_multi_q8_async(a, None, M, K, [dict(w=W, row_begin=row_begin, rows=rows, dst_f32=out)])
    ctx.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("K", [256, 2560])
def test_gemv_bitexact(kqctx, oracle, gtype, M, K):
    rows = 77
    w = synth.gen_weights(gtype, rows, K, seed=10 * gtype + M)
    x = synth.gen_activations(M, K, seed=K + M)
    act = oracle.act_for(gtype, x)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        got = run_q8(kqctx, W, gtype, act, M, K, rows)
    finally:
        W.free()
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"


FULL_RANGE = {kq.TYPE_Q6_K: dict(q6_scales=(-128, 128)), kq.TYPE_Q8_0: dict(q8_quants=(-128, 128))}


@pytest.mark.parametrize("gtype", sorted(FULL_RANGE), ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [1, 2, 4, 8, 9, 40])
@pytest.mark.parametrize("path", [0, 1, 2, 3])
def test_full_range_values_bitexact(kqctx, oracle, gtype, M, path):
    """Q6_K scales over all of int8 (real Q6_K blocks always hold -128 or 127: the quantizer maps
    each block's largest scale there) and Q8_0 quants including -128, on every M > 8 path"""
    if path and M <= 8:
        pytest.skip("the M > 8 path choice does not apply")
    rows, K = 150, 1024
    w = synth.gen_weights(gtype, rows, K, seed=70 + M, **FULL_RANGE[gtype])
    x = synth.gen_activations(M, K, seed=71 + M)
    act = oracle.act_for(gtype, x)
    kqctx.set_option("gemm_path", path)
    W = kqctx.upload(w, gtype, rows, K)
    try:
        got = run_q8(kqctx, W, gtype, act, M, K, rows)
    finally:
        W.free()
        kqctx.set_option("gemm_path", 0)
    ref = oracle.gemm(gtype, w, K, act)
    assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
def test_block_sums_bitexact(kqctx, oracle, gtype):
    """per-super-block integer intermediates (sumi, summ) equal the reference's locals"""
    import torch
    rows, K, M = 19, 1024, 3
    w = synth.gen_weights(gtype, rows, K, seed=3 + gtype)
    x = synth.gen_activations(M, K, seed=4)
    act = oracle.act_for(gtype, x)
    nb = K // (32 if gtype == kq.TYPE_Q8_0 else 256)
    W = kqctx.upload(w, gtype, rows, K)
    si = torch.zeros((M, rows, nb), dtype=torch.int32, device="cuda")
    sm = torch.zeros_like(si)
    out = torch.zeros((M, rows), dtype=torch.float32, device="cuda")
    kqctx.debug_block_sums_async(W, 0, rows, to_dev(act), M, si, sm, out)
    kqctx.synchronize()
    W.free()
    si, sm = si.cpu().numpy(), sm.cpu().numpy()
    for m in range(M):
        for r in range(rows):
            v, rsi, rsm = oracle.vec_dot(gtype, w[r], act[m], K)
            assert np.array_equal(si[m, r], rsi)
            assert np.array_equal(sm[m, r], rsm)
            assert bits(out.cpu().numpy()[m, r]) == bits(v)


@pytest.mark.parametrize("path", golden_files("dot_"), ids=lambda p: p.split("/")[-1][:-4])
def test_reference_golden_through_gpu(kqctx, path):
    """the reference engine's own row-kernel outputs, reproduced by the GPU from the same bytes"""
    g = load_golden(path)
    t, K = int(g["type"]), int(g["K"])
    w, x = g["w"], g["x"]
    rows, M = w.shape[0], x.shape[0]
    # 1) GPU quantizer == reference quantizer (bytes)
    q = kqctx.quantize_q8_0(x) if t == kq.TYPE_Q8_0 else kqctx.quantize_q8k(x)
    assert q.view(np.uint8).reshape(M, -1).tobytes() == g["act"].tobytes()
    # 2) GEMV from the reference's quantized activation == reference fp32 outputs (bits)
    W = kqctx.upload(w, t, rows, K)
    try:
        got = run_q8(kqctx, W, t, g["act"].reshape(-1).view(np.uint8), M, K, rows)
        assert np.array_equal(bits(got), bits(g["out"]))
        # 3) dequant == reference dequant (bits)
        assert np.array_equal(bits(kqctx.dequant_rows(W)), bits(g["dequant"]))
    finally:
        W.free()


def test_fp16_input_path_equals_prequantized(kqctx, oracle):
    """the in-kernel quantization (fp16 input) gives the same result as a pre-quantized input"""
    import torch
    for gtype in TYPES:
        rows, K, M = 50, 2560, 4
        w = synth.gen_weights(gtype, rows, K, seed=gtype)
        x = synth.gen_activations(M, K, seed=99)
        x[1, 256:512] = 0          # all-zero unit (d = 0 path)
        W = kqctx.upload(w, gtype, rows, K)
        out = torch.zeros((M, rows), dtype=torch.float32, device="cuda")
        kqctx.gemm_multi_async(to_dev(x.view(np.uint16)), M, K, [dict(w=W, dst_f32=out)])
        kqctx.synchronize()
        W.free()
        ref = oracle.gemm(gtype, w, K, oracle.act_for(gtype, x))
        assert np.array_equal(bits(out.cpu().numpy()), bits(ref))


def test_dispatch_golden_pinned_outputs(kqctx):
    """the same dispatch with outputs in pinned host memory (written by the kernel in place) and a
    strided fp16 destination; the input stays pageable"""
    import torch
    g = load_golden("dispatch_q4k_q6k")
    K = int(g["K"])
    W0 = kqctx.upload(g["w0"], kq.TYPE_Q4_K, g["w0"].shape[0], K)
    W1 = kqctx.upload(g["w1"], kq.TYPE_Q6_K, g["w1"].shape[0], K)
    M = g["x"].shape[0]
    t0 = torch.full((M, 48), -1.0, dtype=torch.float16).pin_memory()   # stride 48 > 40 rows
    t1 = torch.zeros((M, 24), dtype=torch.float16).pin_memory()
    d0, d1 = t0.numpy(), t1.numpy()
    try:
        kqctx.sdot_gemm_multi_dispatch(g["x"], [dict(w=W0, dst=d0, residual=g["res0"], rows=40), dict(w=W1, dst=d1)])
        assert np.array_equal(bits(d0[:, :40]), bits(g["dst0"]))
        assert np.all(d0[:, 40:] == -1.0)  # the stride padding is untouched
        assert np.array_equal(bits(d1), bits(g["dst1"]))
    finally:
        W0.free()
        W1.free()


def test_dispatch_golden(kqctx):
    """kq_sdot_gemm_multi_dispatch (host pointers) == the reference dispatch's fp16 outputs"""
    g = load_golden("dispatch_q4k_q6k")
    K = int(g["K"])
    W0 = kqctx.upload(g["w0"], kq.TYPE_Q4_K, g["w0"].shape[0], K)
    W1 = kqctx.upload(g["w1"], kq.TYPE_Q6_K, g["w1"].shape[0], K)
    M = g["x"].shape[0]
    d0 = np.zeros((M, 40), np.float16)
    d1 = np.zeros((M, 24), np.float16)
    kqctx.sdot_gemm_multi_dispatch(g["x"], [dict(w=W0, dst=d0, residual=g["res0"]), dict(w=W1, dst=d1)])
    assert np.array_equal(bits(d0), bits(g["dst0"]))
    assert np.array_equal(bits(d1), bits(g["dst1"]))
    # row-level entry points over the dispatch's input (ENG:10986, ENG:3234)
    act = kqctx.quantize_q8k(g["x"])
    from oracle.oracle import Oracle
    o = Oracle()
    for r in (0, 7, 23):
        v = kqctx.eval_single_lm_row_dot(W1, r, 2)
        ref, _, _ = o.vec_dot(kq.TYPE_Q6_K, g["w1"][r], act[2], K)
        assert bits(np.float32(v)) == bits(ref)
        rb = kqctx.sdot_row_batch(W0, r, M)
        refb = o.gemm(kq.TYPE_Q4_K, g["w0"][r:r + 1], K, act)[:, 0]
        assert np.array_equal(bits(rb), bits(refb))
    W0.free()
    W1.free()
    g = load_golden("dispatch_q8_0")
    W = kqctx.upload(g["w"], kq.TYPE_Q8_0, g["w"].shape[0], int(g["K"]))
    d = np.zeros_like(g["dst"])
    kqctx.sdot_gemm_multi_dispatch(g["x"], [dict(w=W, dst=d)])
    W.free()
    assert np.array_equal(bits(d), bits(g["dst"]))


def test_dispatch_strides_row_ranges_and_mtiles(kqctx, oracle):
    """strided outputs, row_begin offsets, 4 tasks, M > 8 (token tiles), fp32 + fp16 outputs"""
    K, M = 512, 11
    x = synth.gen_activations(M, K, 5)
    ws = [synth.gen_weights(t, 64, K, 20 + t) for t in TYPES]
    Ws = [kqctx.upload(w, t, 64, K) for w, t in zip(ws, TYPES)]
    res = synth.gen_activations(M, 70, 6)
    dsts = [np.zeros((M, 70), np.float16) for _ in TYPES]
    f32 = [np.zeros((M, 33), np.float32) for _ in TYPES]
    tasks = [dict(w=W, row_begin=7, rows=33, dst=d, residual=res, dst_f32=f) for W, d, f in zip(Ws, dsts, f32)]
    kqctx.sdot_gemm_multi_dispatch(x, tasks)
    for t, w, d, f in zip(TYPES, ws, dsts, f32):
        ref = oracle.gemm(t, w[7:40], K, oracle.act_for(t, x))
        assert np.array_equal(bits(f), bits(ref))
        ref16 = oracle.epilogue_f16(ref, res[:, :33])
        assert np.array_equal(bits(d[:, :33]), bits(ref16))
        assert not d[:, 33:].any()   # nothing written past the task's rows
    for W in Ws:
        W.free()


def test_config0_shape_bitexact(kqctx, oracle):
    """Benchmark config 0 at full size: Q4_K x Q8_K GEMV, M=1, N=9728, K=2560"""
    N, K = 9728, 2560
    w = synth.gen_weights(kq.TYPE_Q4_K, N, K, seed=1234)
    x = synth.gen_activations(1, K, seed=1235)
    act = oracle.quantize_q8k(x)
    W = kqctx.upload(w, kq.TYPE_Q4_K, N, K)
    got = run_q8(kqctx, W, kq.TYPE_Q4_K, act, 1, K, N)
    W.free()
    ref = oracle.gemm(kq.TYPE_Q4_K, w, K, act)
    assert np.array_equal(bits(got), bits(ref))


def test_dispatch_pinned_input_and_outputs(kqctx, oracle):
    """Host input and outputs in pinned (mapped) memory, the outputs written in place by the
    kernel: bit for bit the oracle on several calls in a row with new input each time, through an
    unaligned input view, and the fp16 + residual epilogue at 2 rows."""
    import torch
    N, K = 9728, 2560
    w = synth.gen_weights(kq.TYPE_Q4_K, N, K, seed=301)
    W = kqctx.upload(w, kq.TYPE_Q4_K, N, K)
    xp = torch.zeros((1, K + 8), dtype=torch.float16).pin_memory().numpy()
    op = torch.zeros((1, N), dtype=torch.float32).pin_memory().numpy()
    tasks = kqctx.make_host_tasks([dict(w=W, dst_f32=op)])
    try:
        for step in range(4):
            x = synth.gen_activations(1, K, seed=310 + step)
            off = 0 if step < 3 else 1  # 2 bytes in: not 16-byte aligned
            xp[:, off:off + K] = x
            kqctx.sdot_gemm_multi_dispatch(xp[:, off:off + K], tasks)
            ref = oracle.gemm(kq.TYPE_Q4_K, w, K, oracle.quantize_q8k(x))
            assert np.array_equal(bits(op), bits(ref)), step
    finally:
        W.free()
    M, N2, K2 = 2, 1000, 512
    w2 = synth.gen_weights(kq.TYPE_Q5_K, N2, K2, seed=320)
    W2 = kqctx.upload(w2, kq.TYPE_Q5_K, N2, K2)
    x2p = torch.zeros((M, K2), dtype=torch.float16).pin_memory().numpy()
    d2p = torch.zeros((M, N2), dtype=torch.float16).pin_memory().numpy()
    res = synth.gen_activations(M, N2, seed=321)
    try:
        for step in range(2):
            x2 = synth.gen_activations(M, K2, seed=322 + step)
            x2p[:] = x2
            kqctx.sdot_gemm_multi_dispatch(x2p, [dict(w=W2, dst=d2p, residual=res)])
            ref = oracle.gemm(kq.TYPE_Q5_K, w2, K2, oracle.quantize_q8k(x2))
            assert np.array_equal(bits(d2p), bits(oracle.epilogue_f16(ref, res))), step
    finally:
        W2.free()


def test_quantizers_bitexact(kqctx, oracle):
    x = synth.gen_activations(6, 2560, 77).astype(np.float32)
    x[1] = 0
    x[2, :300] = 65504.0
    x[3, 5] = -65504.0
    x[4] = 6e-8        # fp16 subnormals
    x = x.astype(np.float16)
    assert kqctx.quantize_q8k(x).tobytes() == oracle.quantize_q8k(x).tobytes()
    assert kqctx.quantize_q8_0(x).tobytes() == oracle.quantize_q8_0(x).tobytes()


def test_error_codes(kqctx):
    w = synth.gen_weights(kq.TYPE_Q4_K, 8, 512, 1)
    with pytest.raises(kq.KQError) as e:
        kqctx.upload(w, 2, 8, 512)          # Q4_0 is not supported
    assert e.value.status == -2
    with pytest.raises(kq.KQError) as e:
        kqctx.upload(w, kq.TYPE_Q4_K, 8, 500)
    assert e.value.status == -3
    W = kqctx.upload(w, kq.TYPE_Q4_K, 8, 512)
    x = synth.gen_activations(1, 256, 1)
    with pytest.raises(kq.KQError) as e:     # K mismatch
        kqctx.sdot_gemm_multi_dispatch(x, [dict(w=W, dst=np.zeros((1, 8), np.float16))])
    assert e.value.status == -3
    x = synth.gen_activations(1, 512, 1)
    with pytest.raises(kq.KQError) as e:     # rows outside the weight
        kqctx.sdot_gemm_multi_dispatch(x, [dict(w=W, row_begin=4, rows=5, dst=np.zeros((1, 8), np.float16))])
    assert e.value.status == -3
    W.free()


def test_bounded_wait_times_out_and_context_survives(kqctx, oracle):
    """failure detection without a GPU fault: a wait on a barrier nothing completes runs out,
    the kernel returns early, the call reports KQ_ERR_TIMEOUT, and the context keeps working"""
    K, rows = 512, 300
    w = synth.gen_weights(kq.TYPE_Q4_K, rows, K, 8)
    x = synth.gen_activations(2, K, 9)
    W = kqctx.upload(w, kq.TYPE_Q4_K, rows, K)
    kqctx.set_option("timeout_us", 2000)
    kqctx.set_option("inject_timeout", 1)
    try:
        with pytest.raises(kq.KQError) as e:
            kqctx.sdot_gemm_multi_dispatch(x, [dict(w=W, dst=np.zeros((2, rows), np.float16))])
        assert e.value.status == -7
    finally:
        kqctx.set_option("inject_timeout", 0)
        kqctx.set_option("timeout_ms", 1000)
    d = np.zeros((2, rows), np.float16)
    kqctx.sdot_gemm_multi_dispatch(x, [dict(w=W, dst=d)])
    W.free()
    ref = oracle.epilogue_f16(oracle.gemm(kq.TYPE_Q4_K, w, K, oracle.quantize_q8k(x)))
    assert np.array_equal(bits(d), bits(ref))


@pytest.mark.parametrize("gtype", TYPES, ids=lambda t: synth.TYPE_NAMES[t])
@pytest.mark.parametrize("M", [3, 16])
def test_edge_activations_fp16_input(kqctx, oracle, gtype, M):
    """fp16 inputs quantized inside the kernels (GEMV at 3 tokens, tensor cores at 16): a row with
    an all-zero super-block (d = 0) and a row holding +-65504 and fp16 subnormals (clamp at +-127,
    tiny products) give the oracle's results -- bit for bit, except Q8_0 rows that the tensor-core
    path sums one 256-value tile at a time (1e-5 of the output scale)"""
    import torch
    from test_gpu_split import check_q80_tolerance
    rows, K = 100, 2560
    w = synth.gen_weights(gtype, rows, K, seed=300 + gtype)
    x = synth.gen_activations(M, K, seed=301 + M)
    x[1, :256] = 0
    x[2, ::7] = np.float16(65504.0)
    x[2, 3::11] = np.float16(-65504.0)
    x[2, 5::13] = np.float16(6e-8)
    W = kqctx.upload(w, gtype, rows, K)
    out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
    try:
        kqctx.gemm_multi_async(to_dev(x.view(np.uint16)), M, K, [dict(w=W, dst_f32=out)])
        kqctx.synchronize()
    finally:
        W.free()
    got = out.cpu().numpy()
    ref = oracle.gemm(gtype, w, K, oracle.act_for(gtype, x))
    if gtype == kq.TYPE_Q8_0 and M > 8:
        check_q80_tolerance(got, ref)
    else:
        assert np.array_equal(bits(got), bits(ref)), f"max |diff| {np.abs(got - ref).max()}"
