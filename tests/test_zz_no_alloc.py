"""kq_lm_head_argmax_noalloc: the LM-head argmax for callers that cannot allocate device memory at
call time (for example a decode loop whose memory is fixed after start-up).  Its scratch is a static
device array shared by all calls; this test checks, through the C ABI, that two calls in a row give
exactly the outputs of the existing entry point kq_lm_head_argmax_async on the same inputs -- the
second call with a smaller best logit than the first, so a scratch array left uncleared between
calls would show up as a wrong argmax.  Kept in its own file, collected last."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev

pytestmark = pytest.mark.gpu


def test_noalloc_lm_head_matches_existing_entry_point_twice(kqctx):
    import torch
    L = kq.load_library()
    f = L.kq_lm_head_argmax_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
    V, K, M = 20000, 2560, 5
    w = synth.gen_weights(kq.TYPE_Q6_K, V, K, seed=901)
    W = kqctx.upload(w, kq.TYPE_Q6_K, V, K)
    x1 = synth.gen_activations(M, K, seed=902)
    x2 = (x1.astype(np.float32) * np.float32(-0.25)).astype(np.float16)   # smaller maxima
    stream = torch.cuda.Stream()
    try:
        for x in (x1, x2):
            xd = to_dev(x.view(np.uint16))
            # existing entry point (context scratch)
            l_ref = torch.zeros((M, V), dtype=torch.float16, device="cuda")
            t_ref = torch.zeros(M, dtype=torch.int32, device="cuda")
            v_ref = torch.zeros(M, dtype=torch.float32, device="cuda")
            kqctx.lm_head_argmax_async(W, xd, M, l_ref, None, t_ref, v_ref)
            kqctx.synchronize()
            # allocation-free entry point (static device scratch)
            l_na = torch.zeros((M, V), dtype=torch.float16, device="cuda")
            t_na = torch.zeros(M, dtype=torch.int32, device="cuda")
            v_na = torch.zeros(M, dtype=torch.float32, device="cuda")
            st = f(W.handle, xd.data_ptr(), M, l_na.data_ptr(), t_na.data_ptr(), v_na.data_ptr(), stream.cuda_stream)
            assert st == 0
            stream.synchronize()
            assert torch.equal(t_na, t_ref)
            assert np.array_equal(bits(v_na.cpu().numpy()), bits(v_ref.cpu().numpy()))
            assert np.array_equal(bits(l_na.cpu().numpy()), bits(l_ref.cpu().numpy()))
        # sizes beyond the static array are refused
        big = torch.zeros((kq_max := 65, K), dtype=torch.float16, device="cuda")
        out = torch.zeros(kq_max, dtype=torch.int32, device="cuda")
        assert f(W.handle, big.data_ptr(), kq_max, None, out.data_ptr(), out.data_ptr(), stream.cuda_stream) == -3
    finally:
        W.free()
