"""kq_lm_head_argmax_noalloc: the LM-head argmax for callers that cannot allocate device memory at
call time (for example a decode loop whose memory is fixed after start-up, or code running inside
another runtime's allocator).  Its scratch is a static device array shared by all calls; these tests
check, through the C ABI, that two calls in a row give the outputs of the existing entry point
kq_lm_head_argmax_async on the same inputs -- the second call with smaller logits than the first,
so a scratch array left uncleared between calls would show up as a wrong argmax:
  * Q6_K at 5, 9, 17 and 64 activation rows (one tile of 8 rows, several tiles, the array's
    maximum): the same bits (both paths are bit-exact to the reference);
  * Q8_0 rows of 4096 values at 3 and 9 rows: logits within the Q8_0 long-row tolerance, and the
    chosen row's logit within that tolerance of the maximum.
Kept in its own file, collected last."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu


def noalloc_fn():
    f = kq.load_library().kq_lm_head_argmax_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    return f


def run_both(kqctx, W, x, V, stream):
    """(existing entry point, allocation-free entry point) -> each (fp16 logits, toks, vals)"""
    import torch
    f = noalloc_fn()
    M = x.shape[0]
    xd = to_dev(x.view(np.uint16))
    outs = []
    for which in ("ctx", "noalloc"):
        lg = torch.zeros((M, V), dtype=torch.float16, device="cuda")
        tk = torch.zeros(M, dtype=torch.int32, device="cuda")
        vl = torch.zeros(M, dtype=torch.float32, device="cuda")
        if which == "ctx":
            kqctx.lm_head_argmax_async(W, xd, M, lg, None, tk, vl)
            kqctx.synchronize()
        else:
            st = f(W.handle, xd.data_ptr(), M, lg.data_ptr(), tk.data_ptr(), vl.data_ptr(), stream.cuda_stream)
            assert st == 0
            stream.synchronize()
        outs.append((lg.cpu().numpy(), tk.cpu().numpy(), vl.cpu().numpy()))
    return outs


@pytest.mark.parametrize("M", [5, 9, 17, 64])
def test_noalloc_lm_head_matches_existing_entry_point_twice(kqctx, M):
    import torch
    V, K = 20000, 2560
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, seed=901)
    W = kqctx.upload(w, kq.TYPE_Q6_K, V, K)
    x1 = synth.gen_activations(M, K, seed=902 + M)
    x2 = (x1.astype(np.float32) * np.float32(-0.25)).astype(np.float16)   # smaller maxima
    stream = torch.cuda.Stream()
    try:
        for x in (x1, x2):
            (l_ref, t_ref, v_ref), (l_na, t_na, v_na) = run_both(kqctx, W, x, V, stream)
            assert np.array_equal(t_na, t_ref)
            assert np.array_equal(bits(v_na), bits(v_ref))
            assert np.array_equal(bits(l_na), bits(l_ref))
        # sizes beyond the static array are refused
        f = noalloc_fn()
        big = torch.zeros((kq_max := 65, K), dtype=torch.float16, device="cuda")
        out = torch.zeros(kq_max, dtype=torch.int32, device="cuda")
        assert f(W.handle, big.data_ptr(), kq_max, None, out.data_ptr(), out.data_ptr(), stream.cuda_stream) == -3
    finally:
        W.free()


@pytest.mark.parametrize("M", [3, 9])
def test_noalloc_lm_head_q8_0_long_rows(kqctx, M):
    """Q8_0 with 4096-value rows: the two entry points may add the block terms in different orders,
    so logits agree within 1e-5 of the output scale plus one fp16 ulp"""
    import torch
    V, K = 6000, 4096
    w = synth.gen_weights(kq.TYPE_Q8_0, V, K, seed=911)
    W = kqctx.upload(w, kq.TYPE_Q8_0, V, K)
    x1 = synth.gen_activations(M, K, seed=912 + M)
    x2 = (x1.astype(np.float32) * np.float32(-0.25)).astype(np.float16)
    stream = torch.cuda.Stream()
    try:
        for x in (x1, x2):
            (l_ref, _, _), (l_na, t_na, v_na) = run_both(kqctx, W, x, V, stream)
            lr, ln = l_ref.astype(np.float32), l_na.astype(np.float32)
            scale = np.abs(lr).max(axis=1, keepdims=True)
            ulp = np.abs(np.spacing(l_ref)).astype(np.float32)
            assert np.all(np.abs(ln - lr) <= 1e-5 * scale + ulp)
            best = lr.max(axis=1)
            chosen = lr[np.arange(M), t_na.astype(np.int64)]
            assert np.all(best - chosen <= 1e-5 * scale[:, 0] + 2 * np.abs(np.spacing(best.astype(np.float16))))
            assert np.array_equal(bits(v_na), bits(ln[np.arange(M), t_na.astype(np.int64)]))
    finally:
        W.free()
