"""GGUF tensor directory (kq_gguf_*, CPU only): parsed from synthetic GGUF v2/v3 images and
files, checked against what the writer put there and against the reference engine's own parser
(parse_gguf_file / find_tensor, ENG:376-420, run from its compiled sources), plus the images it
must reject.  The device upload of the parsed matrices is tested in test_gpu_gguf.py."""
from __future__ import annotations

import os
import struct

import numpy as np
import pytest

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import synth

QTYPES = [kq.TYPE_Q4_K, kq.TYPE_Q5_K, kq.TYPE_Q6_K, kq.TYPE_Q8_0]


def model_image(version=3, alignment=None, seed=0):
    """a small model-like file: quantized matrices of every type, f32/f16 vectors, a 3-D tensor,
    and key/value pairs of every kind the engine skips (strings, u32/u64/f32, string and f32
    arrays including tokenizer.ggml.tokens)"""
    rng = np.random.default_rng(seed)
    tensors = []
    for i, t in enumerate(QTYPES):
        rows, k = 17 + 5 * i, 512 if t != kq.TYPE_Q8_0 else 768
        tensors.append((f"blk.{i}.ffn_{synth.TYPE_NAMES[t]}.weight", t, [k, rows], synth.gen_weights(t, rows, k, seed + i).tobytes()))
    tensors.append(("output_norm.weight", kq.TYPE_F32, [512], rng.standard_normal(512).astype(np.float32).tobytes()))
    tensors.append(("token_embd.weight", kq.TYPE_F16, [256, 3], rng.standard_normal(768).astype(np.float16).tobytes()))
    tensors.append(("blk.0.attn_k.weight", kq.TYPE_Q4_K, [256, 4, 2], synth.gen_weights(kq.TYPE_Q4_K, 8, 256, 9).tobytes()))
    kv = [("general.architecture", synth.GGUF_STRING, "qwen35"),
          ("qwen35.block_count", synth.GGUF_U32, 2),
          ("qwen35.context_length", synth.GGUF_U64, 4096),
          ("qwen35.rope.freq_base", synth.GGUF_F32, 1.0e6),
          ("tokenizer.ggml.tokens", (synth.GGUF_ARRAY, synth.GGUF_STRING), ["<s>", "a", "bc", "été"]),
          ("tokenizer.ggml.scores", (synth.GGUF_ARRAY, synth.GGUF_F32), [0.0, -1.0, -2.5, -3.0])]
    return synth.write_gguf(tensors, kv=kv, version=version, alignment=alignment), tensors


@pytest.mark.parametrize("version,alignment", [(3, None), (2, None), (3, 64), (3, 256)])
def test_directory(version, alignment):
    img, tensors = model_image(version, alignment)
    with kq.Gguf(data=img) as g:
        info = g.info()
        assert info["version"] == version and info["alignment"] == (alignment or 32)
        assert info["data_offset"] % (alignment or 32) == 0
        assert len(g) == len(tensors)
        buf = np.frombuffer(img, np.uint8)
        for i, (name, t, dims, data) in enumerate(tensors):
            r = g.tensor(i)
            assert r["name"] == name and r["type"] == t and r["n_dims"] == len(dims)
            assert r["dims"][:len(dims)] == dims and all(d == 1 for d in r["dims"][len(dims):])
            assert r["n_elems"] == int(np.prod(dims))
            assert r["bytes"] == len(data) and r["offset"] % (alignment or 32) == 0
            assert buf[r["offset"]:r["offset"] + r["bytes"]].tobytes() == data
            assert g.find(name) == i
        assert g.find("blk.9.missing") == -10


@pytest.mark.parametrize("version,alignment", [(3, None), (2, None), (3, 64)])
def test_matches_reference_parser(version, alignment):
    from oracle.oracle import Reference, reference_available
    if not reference_available():
        pytest.skip("reference build (oracle/_ref) not present")
    R = Reference()
    img, tensors = model_image(version, alignment, seed=3)
    ref = R.gguf_parse(img)
    assert ref is not None
    al, do, recs = ref
    with kq.Gguf(data=img) as g:
        info = g.info()
        assert (info["alignment"], info["data_offset"]) == (al, do)
        assert len(g) == len(recs)
        for i, r in enumerate(recs):
            o = g.tensor(i)
            for k in ("name", "n_dims", "dims", "type", "offset", "n_elems", "bytes"):
                assert o[k] == r[k], (i, k, o[k], r[k])
            assert g.find(r["name"]) == R.gguf_find(img, r["name"])
    assert R.gguf_find(img, "nope") == -1


def broken_images():
    img, _ = model_image()
    yield "magic", b"GGUX" + img[4:]
    yield "version1", img[:4] + struct.pack("<I", 1) + img[8:]
    yield "version4", img[:4] + struct.pack("<I", 4) + img[8:]
    for cut in (3, 12, 30, 100, 300, 600):
        yield f"truncated{cut}", img[:cut]
    t = synth.gen_weights(kq.TYPE_Q4_K, 4, 256, 1).tobytes()
    yield "n_dims0", synth.write_gguf([("w", kq.TYPE_Q4_K, [], t)])
    yield "n_dims5", synth.write_gguf([("w", kq.TYPE_Q4_K, [256, 4, 1, 1, 1], t)])
    nested = synth.write_gguf([("w", kq.TYPE_Q4_K, [256, 4], t)], kv=[("x", (synth.GGUF_ARRAY, synth.GGUF_ARRAY), [])])
    yield "nested_array", nested


@pytest.mark.parametrize("name,img", list(broken_images()), ids=lambda v: v if isinstance(v, str) else "")
def test_rejects_malformed(name, img):
    with pytest.raises(kq.KQError) as e:
        kq.Gguf(data=img)
    assert e.value.status == -9  # KQ_ERR_FORMAT
    from oracle.oracle import Reference, reference_available
    if reference_available():
        assert Reference().gguf_parse(img) is None  # the engine refuses them too


def test_rejects_data_past_end():
    """tensor data that runs past the end of the file (the reference does not check this)"""
    img, _ = model_image()
    with pytest.raises(kq.KQError) as e:
        kq.Gguf(data=img[:-100])
    assert e.value.status == -9


def test_open_file(tmp_path):
    img, tensors = model_image(seed=5)
    p = tmp_path / "m.gguf"
    p.write_bytes(img)
    with kq.Gguf(path=str(p)) as g:
        assert len(g) == len(tensors)
        r = g.tensor(1)
        assert r["name"] == tensors[1][0] and r["bytes"] == len(tensors[1][3])
    with pytest.raises(kq.KQError) as e:
        kq.Gguf(path=str(tmp_path / "missing.gguf"))
    assert e.value.status == -10
