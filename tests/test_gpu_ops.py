"""Producers (RMSNorm / SwiGLU + Q8_K), the FFN block, the LM head and dequant on the GPU."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, load_golden, to_dev

pytestmark = pytest.mark.gpu


def ulp_diff16(a, b):
    """distance in fp16 ulps (ordered integer mapping of the bit patterns)"""
    def ordered(x):
        u = bits(np.asarray(x, np.float16)).astype(np.int32)
        return np.where(u & 0x8000, 0x8000 - (u & 0x7FFF), 0x8000 + u)
    return np.abs(ordered(a) - ordered(b))


def test_rmsnorm_matches_reference(kqctx, oracle):
    """fp16 output within 1 ulp of the reference (its fp32 sum of squares is sequential, ours a
    tree sum); the Q8_K of our own fp16 output is bit-exact to the reference quantizer."""
    import torch
    g = load_golden("rmsnorm")
    out = kqctx.rmsnorm_fp16_rows(g["x"], g["gamma"])
    assert ulp_diff16(out, g["out"]).max() <= 1
    assert (bits(out) == bits(g["out"])).mean() > 0.99
    M, K = g["x"].shape
    q = torch.zeros(M * (K // 256) * 292, dtype=torch.uint8, device="cuda")
    o = torch.zeros((M, K), dtype=torch.float16, device="cuda")
    kqctx.rmsnorm_q8k_async(to_dev(g["x"].view(np.uint16)), to_dev(g["gamma"].view(np.uint16)), o, M, K, q)
    kqctx.synchronize()
    o = o.cpu().numpy()
    assert q.cpu().numpy().tobytes() == oracle.quantize_q8k(o).tobytes()


def test_swiglu_matches_reference(kqctx, oracle):
    """CUDA expf vs libm expf: fp16 outputs within 1 ulp, Q8_K of our output bit-exact"""
    import torch
    g = load_golden("swiglu")
    out = kqctx.swiglu_fp16_rows(g["gate"], g["up"])
    assert ulp_diff16(out, g["out"]).max() <= 1
    assert (bits(out) == bits(g["out"])).mean() > 0.99
    M, N = g["gate"].shape
    gd = to_dev(g["gate"].view(np.uint16))
    q = torch.zeros(M * (N // 256) * 292, dtype=torch.uint8, device="cuda")
    kqctx.swiglu_q8k_async(gd, to_dev(g["up"].view(np.uint16)), M, N, q)
    kqctx.synchronize()
    h = gd.cpu().numpy().view(np.float16)
    assert q.cpu().numpy().tobytes() == oracle.quantize_q8k(h).tobytes()


def ffn_check(out, ref, x):
    """FFN tolerance.  The matrix products are bit-exact; the only differences come from the fp32
    rounding of the RMSNorm sum of squares (tree vs sequential order) and of expf (CUDA vs libm),
    each at most 1 fp16 ulp on an intermediate, which can move one quantized activation by one
    step and shift every output of that token slightly.  Required: identical inf/nan positions,
    the residual delta (out - x) within 2e-2 of its max magnitude, and at least half of the fp16
    outputs bit-identical."""
    assert np.array_equal(np.isfinite(out), np.isfinite(ref))
    fin = np.isfinite(ref)
    d_out = (out.astype(np.float32) - x.astype(np.float32))[fin]
    d_ref = (ref.astype(np.float32) - x.astype(np.float32))[fin]
    scale = np.abs(d_ref).max()
    assert np.abs(d_out - d_ref).max() <= 2e-2 * scale
    assert (bits(out) == bits(ref)).mean() >= 0.5


def test_ffn_golden(kqctx):
    g = load_golden("ffn")
    hidden, ffn = int(g["hidden"]), int(g["ffn"])
    Wg = kqctx.upload(g["wg"], kq.TYPE_Q4_K, ffn, hidden)
    Wu = kqctx.upload(g["wu"], kq.TYPE_Q4_K, ffn, hidden)
    Wd = kqctx.upload(g["wd"], kq.TYPE_Q6_K, hidden, ffn)
    out = kqctx.run_ffn(Wg, Wu, Wd, g["x"], g["gamma"])
    for W in (Wg, Wu, Wd):
        W.free()
    ffn_check(out, g["out"], g["x"])


@pytest.mark.parametrize("M", [1, 4, 8, 16])
def test_ffn_tree_verify_shape(kqctx, oracle, M):
    """Benchmark config 2 FFN block (hidden 2560, intermediate 9728): gate/up Q4_K, down Q6_K"""
    hidden, ffn = 2560, 9728
    wg = synth.gen_weights(kq.TYPE_Q4_K, ffn, hidden, 201)
    wu = synth.gen_weights(kq.TYPE_Q4_K, ffn, hidden, 202)
    wd = synth.gen_weights(kq.TYPE_Q6_K, hidden, ffn, 203)
    x = synth.gen_activations(M, hidden, 204)
    # RMSNorm weights of ~0.1 keep the random-weight FFN inside the fp16 range
    gamma = (synth.gen_gamma(hidden, 205).astype(np.float32) * 0.1).astype(np.float16)
    Wg = kqctx.upload(wg, kq.TYPE_Q4_K, ffn, hidden)
    Wu = kqctx.upload(wu, kq.TYPE_Q4_K, ffn, hidden)
    Wd = kqctx.upload(wd, kq.TYPE_Q6_K, hidden, ffn)
    out = kqctx.run_ffn(Wg, Wu, Wd, x, gamma)
    for W in (Wg, Wu, Wd):
        W.free()
    ref = oracle.ffn(wg, kq.TYPE_Q4_K, wu, kq.TYPE_Q4_K, wd, kq.TYPE_Q6_K, hidden, ffn, x, gamma)
    ffn_check(out, ref, x)


@pytest.mark.parametrize("M", [1, 16])
def test_ffn_block_as_one_graph(M):
    """kq_run_ffn_async (RMSNorm+Q8_K, gate/up, SwiGLU+Q8_K, down+residual: four launches linked by
    programmatic dependent launch) captured once into a CUDA graph after an eager call has sized
    its scratch; two replays give the eager call's bits (GEMV path at 1 token, tensor cores at 16)"""
    import torch
    hidden, ffn = 2560, 9728
    wg = synth.gen_weights(kq.TYPE_Q4_K, ffn, hidden, 211)
    wu = synth.gen_weights(kq.TYPE_Q4_K, ffn, hidden, 212)
    wd = synth.gen_weights(kq.TYPE_Q6_K, hidden, ffn, 213)
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
        finally:
            del g
            torch.cuda.synchronize()
            for W in Ws:
                W.free()


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
