"""libkq.so loads, exports exactly what include/*.h declare, and its host-side logic works
without a GPU (no compute calls here)."""
from __future__ import annotations

import ctypes as C
import os
import re

import pytest

from conftest import ROOT

import npu880_mtk_npu_llm_runtime_b200 as kq
from npu880_mtk_npu_llm_runtime_b200 import build as kqbuild


@pytest.fixture(scope="module")
def lib():
    kqbuild.build()
    return kq.load_library()


def header_symbols():
    """every function declared in include/*.h"""
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(kq_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_header_declares_the_python_export_list():
    assert header_symbols() == sorted(kq.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in header_symbols():
        assert hasattr(lib, name), f"libkq.so does not export {name}"


def test_exports_are_c_symbols():
    out = os.popen(f"nm -D --defined-only {kq.LIB_PATH}").read()
    defined = set(re.findall(r" T (kq_[a-z0-9_]+)$", out, flags=re.M))
    assert set(header_symbols()) <= defined


def test_row_bytes_matches_compute_ggml_bytes(lib):
    # ENG:364-374
    assert lib.kq_row_bytes(12, 2560) == 1440
    assert lib.kq_row_bytes(13, 2560) == 1760
    assert lib.kq_row_bytes(14, 9728) == 7980
    assert lib.kq_row_bytes(8, 2560) == 2720
    assert lib.kq_row_bytes(0, 10) == 40
    assert lib.kq_row_bytes(1, 10) == 20
    assert lib.kq_row_bytes(99, 2560) == 0


def test_status_strings(lib):
    for code in kq.STATUS:
        assert lib.kq_status_string(code)
    assert lib.kq_status_string(-7) == b"device-side wait timed out"


def test_init_without_device_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    h = C.c_void_p()
    assert lib.kq_init(0, C.byref(h)) == -6      # KQ_ERR_NO_DEVICE, no abort
    assert h.value is None
    with pytest.raises(kq.KQError):
        kq.Context(0)


def test_null_arguments_rejected(lib):
    assert lib.kq_init(0, None) == -1
    assert lib.kq_destroy(None) == -1
    assert lib.kq_weight_free(None, None) == -1
    assert lib.kq_synchronize(None) == -1
    assert lib.kq_last_error(None) == b"no context"


def test_synth_layouts():
    from npu880_mtk_npu_llm_runtime_b200 import synth
    from oracle.oracle import Oracle
    o = Oracle()
    for t in (8, 12, 13, 14):
        w = synth.gen_weights(t, 3, 512, 1)
        assert w.shape == (3, o.row_bytes(t, 512))
    # scale/min packing inverts get_scale_min_k4 (ENG:743-749)
    import numpy as np
    rng = np.random.default_rng(0)
    sc = rng.integers(0, 64, size=(5, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(5, 8), dtype=np.uint8)
    packed = synth.pack_scale_min_k4(sc, mn)
    lib = o.L
    for b in range(5):
        for j in range(8):
            d = C.c_uint8()
            m = C.c_uint8()
            lib.kqo_get_scale_min_k4(j, packed[b].ctypes.data_as(C.c_void_p), C.byref(d), C.byref(m))
            assert (d.value, m.value) == (sc[b, j], mn[b, j])


def test_peer_gather_struct_layout(tmp_path):
    """kq_peer_gather as compiled by C has the field offsets of the ctypes mirror."""
    import subprocess
    src = tmp_path / "layout.c"
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "kq.h"\nint main(void) {\n'
                   '  printf("%zu %zu %zu %zu %zu %zu %zu\\n", offsetof(kq_peer_gather, world), offsetof(kq_peer_gather, rank),\n'
                   '         offsetof(kq_peer_gather, M), offsetof(kq_peer_gather, row_stride),\n'
                   '         offsetof(kq_peer_gather, row_begin), offsetof(kq_peer_gather, regions), sizeof(kq_peer_gather));\n'
                   '  return 0;\n}\n')
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.check_call(["gcc", "-I", inc, str(src), "-o", str(exe)])
    got = [int(v) for v in subprocess.check_output([str(exe)]).split()]
    S = kq.PeerGatherStruct
    want = [S.world.offset, S.rank.offset, S.M.offset, S.row_stride.offset, S.row_begin.offset, S.regions.offset,
            C.sizeof(S)]
    assert got == want


def test_peer_region_bytes(lib):
    """256 bytes of control words, then two buffers of [M][row_stride] 64-bit entries"""
    assert lib.kq_peer_region_bytes(2, 151936) == 256 + 2 * 2 * 151936 * 8
    assert lib.kq_peer_region_bytes(0, 151936) == 0


def test_every_option_is_documented():
    """each option name kq_set_option accepts is described in the header's option list"""
    api = open(os.path.join(ROOT, "npu880_mtk_npu_llm_runtime_b200", "csrc", "kq_api.cu")).read()
    accepted = set(re.findall(r'strcmp\(name, "([a-z0-9_]+)"\)', api))
    header = open(os.path.join(ROOT, "include", "kq.h")).read()
    doc = header[header.index("/* Options:"):header.index("int kq_set_option(")]
    assert accepted, "no option names found"
    missing = sorted(o for o in accepted if f'"{o}"' not in doc)
    assert not missing, f"options accepted but not documented in kq.h: {missing}"
