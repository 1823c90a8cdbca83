"""Device weights from a GGUF file: kq_gguf_upload_all uploads every quantized matrix of a
synthetic model file (f32 / f16 vectors and a 3-D tensor stay NULL), kq_gguf_upload takes one by
name, and products over the uploaded weights are bit-exact against the oracle on the file's own
bytes -- the path the engine takes from its mmap (init_sdot_task, ENG:4163-4181)."""
from __future__ import annotations

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth
from conftest import bits, to_dev
from test_gguf import QTYPES, model_image

pytestmark = pytest.mark.gpu


def test_upload_all_and_products(kqctx, oracle, tmp_path):
    import torch
    img, tensors = model_image(alignment=64, seed=11)
    p = tmp_path / "model.gguf"
    p.write_bytes(img)
    M = 3
    with kq.Gguf(path=str(p)) as g:
        ws = g.upload_all(kqctx)
        try:
            assert [w is not None for w in ws] == [True] * len(QTYPES) + [False, False, False]
            for i, (name, t, dims, data) in enumerate(tensors[:len(QTYPES)]):
                W = ws[i]
                K, rows = dims
                assert (W.type, W.rows, W.cols) == (t, rows, K)
                x = synth.gen_activations(M, K, seed=20 + i)
                act = oracle.act_for(t, x)
                out = torch.full((M, rows), float("nan"), dtype=torch.float32, device="cuda")
                a = to_dev(act)
                kqctx.gemm_multi_q8_async(None if t == kq.TYPE_Q8_0 else a, a if t == kq.TYPE_Q8_0 else None, M, K,
                                          [dict(w=W, dst_f32=out)])
                kqctx.synchronize()
                wrows = np.frombuffer(data, np.uint8).reshape(rows, -1)
                ref = oracle.gemm(t, wrows, K, act)
                got = out.cpu().numpy()
                assert np.array_equal(bits(got), bits(ref)), f"{name}: max |diff| {np.abs(got - ref).max()}"
        finally:
            for w in ws:
                if w is not None:
                    w.free()
        # one matrix by name, through the blocking dispatch with host buffers
        idx = g.find("blk.2.ffn_q6_k.weight")
        W = g.upload(kqctx, idx)
        try:
            K, rows = tensors[idx][2]
            x = synth.gen_activations(2, K, seed=31)
            dst = np.zeros((2, rows), np.float16)
            kqctx.sdot_gemm_multi_dispatch(x, [dict(w=W, dst=dst)])
            ref = oracle.epilogue_f16(oracle.gemm(kq.TYPE_Q6_K, np.frombuffer(tensors[idx][3], np.uint8).reshape(rows, -1),
                                                  K, oracle.quantize_q8k(x)))
            assert np.array_equal(bits(dst), bits(ref))
        finally:
            W.free()
        with pytest.raises(kq.KQError) as e:  # an f32 vector is not a quantized matrix
            g.upload(kqctx, g.find("output_norm.weight"))
        assert e.value.status == -2
