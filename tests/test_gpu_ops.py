"""Producers (RMSNorm / SwiGLU + Q8_K), the FFN block, the LM head and dequant on the GPU."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import all_fp16_gate, bits, load_golden, rmsnorm_cases, to_dev

pytestmark = pytest.mark.gpu


def test_rmsnorm_bitexact(kqctx, oracle):
    """rmsnorm_fp16_rows_fast (ENG:4264-4314): fp16 outputs and their Q8_K bit for bit -- the fp32
    sum of squares in the reference's sequential order (golden fixture from the compiled
    reference, then seeded cases checked against the oracle)"""
    import torch
    g = load_golden("rmsnorm")
    out = kqctx.rmsnorm_fp16_rows(g["x"], g["gamma"])
    assert np.array_equal(bits(out), bits(g["out"]))
    for M, K, x, gamma in rmsnorm_cases():
        ref, refq = oracle.rmsnorm(x, gamma)
        q = torch.zeros(M * (K // 256) * 292, dtype=torch.uint8, device="cuda")
        o = torch.zeros((M, K), dtype=torch.float16, device="cuda")
        kqctx.rmsnorm_q8k_async(to_dev(x.view(np.uint16)), to_dev(gamma.view(np.uint16)), o, M, K, q)
        kqctx.synchronize()
        o = o.cpu().numpy()
        assert np.array_equal(bits(o), bits(ref)), (M, K)
        fin = np.isfinite(ref).all(axis=1)
        qb = q.cpu().numpy().reshape(M, -1)
        assert np.array_equal(qb[fin], refq.view(np.uint8).reshape(M, -1)[fin]), (M, K)


def _libm_expf():
    import ctypes
    f = ctypes.CDLL("libm.so.6").expf
    f.restype, f.argtypes = ctypes.c_float, [ctypes.c_float]
    return f


@pytest.mark.parametrize("up_kind", ["ones", "random"])
def test_swiglu_exhaustive_fp16_gate(kqctx, oracle, up_kind):
    """swiglu_fp16_rows_fast (ENG:4326-4383) over all 65,536 fp16 gate values: fp16 outputs bit for
    bit equal to the reference's scalar loop with the C library's expf (NaN where it gives NaN),
    and Q8_K of every all-finite row bit-exact; host and device entry points"""
    import torch
    gate = all_fp16_gate(256)
    rng = np.random.default_rng(5)
    up = (np.ones((256, 256), np.float16) if up_kind == "ones"
          else (rng.standard_normal((256, 256)) * 2.0).astype(np.float16))
    ref, refq = oracle.swiglu(gate, up)
    nan = np.isnan(ref)
    out = kqctx.swiglu_fp16_rows(gate, up)
    assert np.array_equal(np.isnan(out), nan)
    assert np.array_equal(bits(out)[~nan], bits(ref)[~nan])
    gd = to_dev(gate.view(np.uint16))
    q = torch.zeros(256 * 292, dtype=torch.uint8, device="cuda")
    kqctx.swiglu_q8k_async(gd, to_dev(up.view(np.uint16)), 256, 256, q)
    kqctx.synchronize()
    h = gd.cpu().numpy().view(np.float16)
    assert np.array_equal(bits(h)[~nan], bits(ref)[~nan])
    fin = np.isfinite(ref).all(axis=1)
    assert fin.sum() > 200
    assert np.array_equal(q.cpu().numpy().reshape(256, -1)[fin], refq.view(np.uint8).reshape(256, -1)[fin])


def test_swiglu_gpu_exp_option(kqctx, oracle):
    """option swiglu_exp = 1 (exp in fp64 on the GPU, rounded once): differs from the C library only
    where the library's expf is not the correctly rounded value"""
    expf = _libm_expf()
    gate = all_fp16_gate(256)
    up = np.ones((256, 256), np.float16)
    ref, _ = oracle.swiglu(gate, up)
    g32 = gate.astype(np.float32).ravel()
    fin = np.isfinite(g32)
    cr = np.exp(-g32.astype(np.float64)).astype(np.float32)
    lib = np.array([expf(float(-v)) if f else 0.0 for v, f in zip(g32, fin)], np.float32)
    differ = fin & (cr.view(np.uint32) != lib.view(np.uint32))
    with kq.Context(0) as ctx:
        ctx.set_option("swiglu_exp", 1)
        out = ctx.swiglu_fp16_rows(gate, up)
    nan = np.isnan(ref).ravel()
    mism = (bits(out).ravel() != bits(ref).ravel()) & ~nan
    assert not np.any(mism & ~differ)


def ffn_check(out, ref):
    """The FFN block is bit-exact: every product is, RMSNorm sums in the reference's order and
    SwiGLU uses the reference's expf (fp16 outputs compared bit for bit, NaN positions equal)."""
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    ok = ~np.isnan(ref)
    mism = int((bits(out)[ok] != bits(ref)[ok]).sum())
    assert mism == 0, f"{mism} of {ok.sum()} fp16 outputs differ"


def test_ffn_golden(kqctx):
    g = load_golden("ffn")
    hidden, ffn = int(g["hidden"]), int(g["ffn"])
    Wg = kqctx.upload(g["wg"], kq.TYPE_Q4_K, ffn, hidden)
    Wu = kqctx.upload(g["wu"], kq.TYPE_Q4_K, ffn, hidden)
    Wd = kqctx.upload(g["wd"], kq.TYPE_Q6_K, hidden, ffn)
    out = kqctx.run_ffn(Wg, Wu, Wd, g["x"], g["gamma"])
    for W in (Wg, Wu, Wd):
        W.free()
    ffn_check(out, g["out"])


@pytest.fixture(scope="module")
def cfg2_weights():
    hidden, ffn = 2560, 9728
    return (synth.gen_weights(kq.TYPE_Q4_K, ffn, hidden, 201), synth.gen_weights(kq.TYPE_Q4_K, ffn, hidden, 202),
            synth.gen_weights(kq.TYPE_Q6_K, hidden, ffn, 203))


@pytest.mark.parametrize("M", [1, 4, 8, 16, 32, 64])
def test_ffn_tree_verify_shape(kqctx, oracle, cfg2_weights, M):
    """Benchmark config 2 FFN block (hidden 2560, intermediate 9728; gate/up Q4_K, down Q6_K) at
    every draft-token count of the config, bit-exact to the reference's SDOT FFN sequence
    (ENG:8283-8298) restated by the oracle"""
    hidden, ffn = 2560, 9728
    wg, wu, wd = cfg2_weights
    x = synth.gen_activations(M, hidden, 204 + M)
    # RMSNorm weights of ~0.1 keep the random-weight FFN inside the fp16 range
    gamma = (synth.gen_gamma(hidden, 205).astype(np.float32) * 0.1).astype(np.float16)
    Wg = kqctx.upload(wg, kq.TYPE_Q4_K, ffn, hidden)
    Wu = kqctx.upload(wu, kq.TYPE_Q4_K, ffn, hidden)
    Wd = kqctx.upload(wd, kq.TYPE_Q6_K, hidden, ffn)
    out = kqctx.run_ffn(Wg, Wu, Wd, x, gamma)
    for W in (Wg, Wu, Wd):
        W.free()
    ref = oracle.ffn(wg, kq.TYPE_Q4_K, wu, kq.TYPE_Q4_K, wd, kq.TYPE_Q6_K, hidden, ffn, x, gamma)
    ffn_check(out, ref)


@pytest.mark.parametrize("M", [1, 16])
def test_ffn_block_as_one_graph(kqctx, oracle, cfg2_weights, M):
    """kq_run_ffn_async (RMSNorm+Q8_K, gate/up, SwiGLU+Q8_K, down+residual: four launches linked by
    programmatic dependent launch) captured once into a CUDA graph after an eager call has sized
    its scratch; two replays give the eager call's bits and the oracle's (GEMV path at 1 token,
    tensor cores at 16)"""
    import torch
    hidden, ffn = 2560, 9728
    wg, wu, wd = cfg2_weights
    x16 = synth.gen_activations(M, hidden, 214)
    gamma = (synth.gen_gamma(hidden, 215).astype(np.float32) * 0.1).astype(np.float16)
    s = torch.cuda.Stream()
    with kq.Context(0) as ctx:  # its own context: the session context keeps its stream
        ctx.set_stream(s.cuda_stream)
        Ws = [ctx.upload(wg, kq.TYPE_Q4_K, ffn, hidden), ctx.upload(wu, kq.TYPE_Q4_K, ffn, hidden),
              ctx.upload(wd, kq.TYPE_Q6_K, hidden, ffn)]
        x = to_dev(x16.view(np.uint16))
        gm = to_dev(gamma.view(np.uint16))
        eager = torch.zeros((M, hidden), dtype=torch.float16, device="cuda")
        outg = torch.zeros((M, hidden), dtype=torch.float16, device="cuda")
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.stream(s):
                ctx.run_ffn_async(*Ws, M, x, gm, eager)
            ctx.synchronize()
            with torch.cuda.graph(g, stream=s):
                ctx.run_ffn_async(*Ws, M, x, gm, outg)
            want = bits(eager.cpu().numpy())
            for _ in range(2):
                with torch.cuda.stream(s):
                    outg.fill_(float("nan"))
                    g.replay()
                ctx.synchronize()
                assert np.array_equal(bits(outg.cpu().numpy()), want)
            # scratch the graph recorded must not be freed: growing it is refused until released
            with pytest.raises(kq.KQError):
                ctx.run_ffn_async(*Ws, 2 * M + 8, to_dev(np.zeros((2 * M + 8) * hidden, np.uint16)), gm,
                                  torch.zeros((2 * M + 8, hidden), dtype=torch.float16, device="cuda"))
        finally:
            del g
            torch.cuda.synchronize()
            ctx.set_option("graph_released", 1)
            for W in Ws:
                W.free()
    ref = oracle.ffn(wg, kq.TYPE_Q4_K, wu, kq.TYPE_Q4_K, wd, kq.TYPE_Q6_K, hidden, ffn, x16, gamma)
    ffn_check(eager.cpu().numpy(), ref)


def test_lm_head_golden_and_argmax(kqctx, oracle):
    g = load_golden("lm_head_q6k")
    K = int(g["K"])
    W = kqctx.upload(g["w"], kq.TYPE_Q6_K, g["w"].shape[0], K)
    toks, vals, logits = kqctx.lm_head_argmax(W, g["x"])
    W.free()
    assert np.array_equal(bits(logits), bits(g["logits"]))
    ref = np.argmax(g["logits"].astype(np.float32), axis=1)
    assert np.array_equal(toks.astype(np.int64), ref)
    assert np.array_equal(vals, g["logits"].astype(np.float32)[np.arange(len(ref)), ref])


def test_lm_head_ties_pick_first_row(kqctx, oracle):
    """duplicate rows give equal logits: the first (lowest) row id wins, like the strict '>' scan"""
    K, V = 512, 5000
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, 31)
    x = synth.gen_activations(3, K, 32)
    act = oracle.quantize_q8k(x)
    best, _, _ = oracle.rows_argmax(kq.TYPE_Q6_K, w, K, act, f16_compare=True)
    w2 = w.copy()
    w2[4000] = w[best[0]]
    w2[best[0] + 1:4000][:1] = w[best[0]]   # another duplicate just after the winner
    W = kqctx.upload(w2, kq.TYPE_Q6_K, V, K)
    toks, vals, _ = kqctx.lm_head_argmax(W, x, want_logits=False)
    W.free()
    rb, rv, _ = oracle.rows_argmax(kq.TYPE_Q6_K, w2, K, act, f16_compare=True)
    assert np.array_equal(toks, rb) and np.array_equal(bits(vals), bits(rv))


@pytest.mark.parametrize("M", [12, 40])
@pytest.mark.parametrize("want_logits", [True, False], ids=["logits", "no-logits"])
@pytest.mark.parametrize("V", [5000, 4999])
def test_lm_head_many_tokens(kqctx, oracle, M, want_logits, V):
    """more than 8 tokens: fp16 logits from the matrix-product path, then one scan of them (8 per
    16-byte load when the vocabulary is a multiple of 8, else one by one) -- the same tokens,
    values and first-row-on-ties rule as the fused GEMV argmax; a duplicated winning row checks
    the tie rule"""
    K = 512
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, 41)
    x = synth.gen_activations(M, K, 42)
    act = oracle.quantize_q8k(x)
    best, _, _ = oracle.rows_argmax(kq.TYPE_Q6_K, w, K, act, f16_compare=True)
    w2 = w.copy()
    w2[V - 1] = w[best[0]]   # an equal logit later in the vocabulary: the first row must win
    W = kqctx.upload(w2, kq.TYPE_Q6_K, V, K)
    toks, vals, logits = kqctx.lm_head_argmax(W, x, want_logits=want_logits)
    W.free()
    rb, rv, ref = oracle.rows_argmax(kq.TYPE_Q6_K, w2, K, act, f16_compare=True, want_logits=True)
    assert np.array_equal(toks, rb) and np.array_equal(bits(vals), bits(rv))
    if want_logits:
        assert np.array_equal(bits(logits), bits(ref.astype(np.float16)))


def test_lm_head_config1_shape(kqctx, oracle):
    """Benchmark config 1 at full size: Q6_K LM head, N=151936, K=2560 (logits bit-exact)"""
    import torch
    V, K = 151936, 2560
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, 4321)
    x = synth.gen_activations(1, K, 4322)
    W = kqctx.upload(w, kq.TYPE_Q6_K, V, K)
    lf = torch.zeros((1, V), dtype=torch.float32, device="cuda")
    tk = torch.zeros(1, dtype=torch.int32, device="cuda")
    tv = torch.zeros(1, dtype=torch.float32, device="cuda")
    kqctx.lm_head_argmax_async(W, to_dev(x.view(np.uint16)), 1, None, lf, tk, tv)
    kqctx.synchronize()
    W.free()
    act = oracle.quantize_q8k(x)
    rb, rv, ref = oracle.rows_argmax(kq.TYPE_Q6_K, w, K, act, f16_compare=True, want_logits=True)
    assert np.array_equal(bits(lf.cpu().numpy()), bits(ref))
    assert int(tk.item()) == int(rb[0])


def test_indexed_rows_argmax(kqctx, oracle):
    """eval_indexed_ext_lm_rows_parallel: gathered rows, fp32 comparison, in-place merge"""
    K, V = 2560, 3000
    w = synth.gen_weights(kq.TYPE_Q4_K, V, K, 41)
    x = synth.gen_activations(1, K, 42)
    W = kqctx.upload(w, kq.TYPE_Q4_K, V, K)
    kqctx.quantize_q8k(x)                   # makes x the context's current input
    rng = np.random.default_rng(43)
    ids = rng.choice(V, size=700, replace=False).astype(np.uint32)
    logits = np.full(V, np.float16(-100.0), dtype=np.float16)
    toks, vals = kqctx.eval_indexed_rows_argmax(W, ids, 1, logits_m1=logits)
    act = oracle.quantize_q8k(x)
    rb, rv, rl = oracle.rows_argmax(kq.TYPE_Q4_K, w, K, act, row_ids=ids, want_logits=True)
    assert toks[0] == rb[0] and bits(vals[0]) == bits(rv[0])
    assert np.array_equal(bits(logits[ids]), bits(rl[0].astype(np.float16)))
    mask = np.ones(V, bool)
    mask[ids] = False
    assert np.all(logits[mask] == np.float16(-100.0))
    # a running best that beats every listed row is kept
    t2, v2 = kqctx.eval_indexed_rows_argmax(W, ids, 1, top_toks=np.array([7], np.uint32),
                                            top_vals=np.array([1e9], np.float32))
    assert t2[0] == 7 and v2[0] == np.float32(1e9)
    W.free()


@pytest.mark.parametrize("gtype", [kq.TYPE_Q4_K, kq.TYPE_Q5_K, kq.TYPE_Q6_K, kq.TYPE_Q8_0],
                         ids=lambda t: synth.TYPE_NAMES[t])
def test_dequant_bitexact(kqctx, oracle, gtype):
    w = synth.gen_weights(gtype, 33, 768, 50 + gtype)
    W = kqctx.upload(w, gtype, 33, 768)
    got = kqctx.dequant_rows(W, 3, 20)
    W.free()
    assert np.array_equal(bits(got), bits(oracle.dequant(gtype, w[3:23], 768)))
