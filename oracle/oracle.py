"""ctypes front-end of the parity checker (TEST INFRASTRUCTURE ONLY).

Wraps two libraries built by oracle/Makefile:

* ``libkq_oracle.so`` -- the C restatement of the reference's scalar K-quant path
  (kq_oracle.c), always available;
* ``_ref/libkqref.so`` -- the unmodified reference engine compiled from its own sources
  (ref_harness.c), available where it was built.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm import this
module; the product package never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "libkq_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkqref.so")

TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 8, 12, 13, 14

# BlockQ8K (ENG:868-872) and BlockQ8_0_Fast (ENG:874-877) as numpy records
Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsum32", "<i4", (8,))])
Q8_0_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (32,))])
assert Q8K_DTYPE.itemsize == 292 and Q8_0_DTYPE.itemsize == 36

_vp = C.c_void_p


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def build(quiet: bool = True) -> None:
    """Build libkq_oracle.so (and _ref/libkqref.so when the reference sources are present)."""
    out = subprocess.run(["make", "-s", "-f", os.path.join(HERE, "Makefile")],
                         capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout, end="")


class Oracle:
    """The C restatement (kq_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.L = L
        L.kqo_row_bytes.restype = C.c_uint64
        L.kqo_row_bytes.argtypes = [C.c_uint32, C.c_uint64]
        L.kqo_quantize_row_q8k.argtypes = [_vp, _vp, C.c_int]
        L.kqo_quantize_row_q8_0.argtypes = [_vp, _vp, C.c_int]
        L.kqo_vec_dot.restype = C.c_float
        L.kqo_vec_dot.argtypes = [C.c_uint32, _vp, _vp, C.c_int, _vp, _vp]
        L.kqo_gemm.argtypes = [C.c_uint32, _vp, C.c_size_t, C.c_int, C.c_int, _vp, C.c_int, _vp, C.c_size_t]
        L.kqo_epilogue_f16.argtypes = [_vp, C.c_size_t, C.c_int, C.c_int, _vp, C.c_size_t, _vp, C.c_size_t]
        L.kqo_dequant_row.argtypes = [C.c_uint32, _vp, C.c_int, _vp]
        L.kqo_rmsnorm_rows.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, _vp]
        L.kqo_swiglu_rows.argtypes = [_vp, _vp, C.c_int, C.c_int, _vp]
        L.kqo_ffn.argtypes = [C.c_uint32, _vp, C.c_uint32, _vp, C.c_uint32, _vp, C.c_int, C.c_int,
                              _vp, _vp, _vp, C.c_int]
        L.kqo_rows_argmax.argtypes = [C.c_uint32, _vp, C.c_size_t, C.c_int, _vp, C.c_int, _vp, C.c_int,
                                      C.c_int, _vp, _vp, _vp]

    def row_bytes(self, gtype: int, k: int) -> int:
        return int(self.L.kqo_row_bytes(gtype, k))

    def quantize_q8k(self, x16: np.ndarray) -> np.ndarray:
        """fp16 [M, K] -> BlockQ8K [M, K/256]"""
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros((M, K // 256), dtype=Q8K_DTYPE)
        for m in range(M):
            self.L.kqo_quantize_row_q8k(_ptr(x16[m]), _ptr(out[m]), K)
        return out

    def quantize_q8_0(self, x16: np.ndarray) -> np.ndarray:
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros((M, K // 32), dtype=Q8_0_DTYPE)
        for m in range(M):
            self.L.kqo_quantize_row_q8_0(_ptr(x16[m]), _ptr(out[m]), K)
        return out

    def act_for(self, gtype: int, x16: np.ndarray) -> np.ndarray:
        return self.quantize_q8_0(x16) if gtype == TYPE_Q8_0 else self.quantize_q8k(x16)

    def vec_dot(self, gtype: int, w_row: np.ndarray, act_row: np.ndarray, k: int):
        """-> (fp32 result, sumi[nb], summ[nb])"""
        nb = k // (32 if gtype == TYPE_Q8_0 else 256)
        sumi = np.zeros(nb, dtype=np.int32)
        summ = np.zeros(nb, dtype=np.int32)
        v = self.L.kqo_vec_dot(gtype, _ptr(np.ascontiguousarray(w_row)), _ptr(np.ascontiguousarray(act_row)),
                               k, _ptr(sumi), _ptr(summ))
        return np.float32(v), sumi, summ

    def gemm(self, gtype: int, w: np.ndarray, k: int, act: np.ndarray) -> np.ndarray:
        """w uint8[rows, row_bytes], act [M, nb] -> fp32 [M, rows]"""
        rows = w.shape[0]
        M = act.shape[0]
        out = np.zeros((M, rows), dtype=np.float32)
        self.L.kqo_gemm(gtype, _ptr(np.ascontiguousarray(w)), w.shape[1], rows, k,
                        _ptr(np.ascontiguousarray(act)), M, _ptr(out), rows)
        return out

    def epilogue_f16(self, sums: np.ndarray, residual: np.ndarray | None = None) -> np.ndarray:
        M, rows = sums.shape
        out = np.zeros((M, rows), dtype=np.float16)
        res = None if residual is None else np.ascontiguousarray(residual, dtype=np.float16)
        self.L.kqo_epilogue_f16(_ptr(np.ascontiguousarray(sums, dtype=np.float32)), rows, rows, M,
                                _ptr(out), rows, _ptr(res), 0 if res is None else res.shape[1])
        return out

    def dequant(self, gtype: int, w: np.ndarray, k: int) -> np.ndarray:
        rows = w.shape[0]
        out = np.zeros((rows, k), dtype=np.float16)
        for r in range(rows):
            self.L.kqo_dequant_row(gtype, _ptr(np.ascontiguousarray(w[r])), k, _ptr(out[r]))
        return out

    def rmsnorm(self, x16: np.ndarray, gamma: np.ndarray):
        """-> (fp16 normalised rows, BlockQ8K of them)"""
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros_like(x16)
        q = np.zeros((M, K // 256), dtype=Q8K_DTYPE)
        self.L.kqo_rmsnorm_rows(_ptr(x16), _ptr(np.ascontiguousarray(gamma, dtype=np.float16)),
                                _ptr(out), M, K, _ptr(q))
        return out, q

    def swiglu(self, gate: np.ndarray, up: np.ndarray):
        g = np.array(gate, dtype=np.float16, copy=True, order="C")
        M, N = g.shape
        q = np.zeros((M, N // 256), dtype=Q8K_DTYPE)
        self.L.kqo_swiglu_rows(_ptr(g), _ptr(np.ascontiguousarray(up, dtype=np.float16)), M, N, _ptr(q))
        return g, q

    def ffn(self, wg, tg, wu, tu, wd, td, hidden, ffn, x16, gamma):
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M = x16.shape[0]
        out = np.zeros_like(x16)
        self.L.kqo_ffn(tg, _ptr(np.ascontiguousarray(wg)), tu, _ptr(np.ascontiguousarray(wu)),
                       td, _ptr(np.ascontiguousarray(wd)), hidden, ffn, _ptr(x16),
                       _ptr(np.ascontiguousarray(gamma, dtype=np.float16)), _ptr(out), M)
        return out

    def rows_argmax(self, gtype, w, k, act, row_ids=None, f16_compare=False, want_logits=False):
        M = act.shape[0]
        ids = None if row_ids is None else np.ascontiguousarray(row_ids, dtype=np.uint32)
        n = w.shape[0] if ids is None else ids.shape[0]
        logits = np.zeros((M, n), dtype=np.float32) if want_logits else None
        bi = np.zeros(M, dtype=np.uint32)
        bv = np.zeros(M, dtype=np.float32)
        self.L.kqo_rows_argmax(gtype, _ptr(np.ascontiguousarray(w)), w.shape[1], k, _ptr(ids), n,
                               _ptr(np.ascontiguousarray(act)), M, int(bool(f16_compare)),
                               _ptr(logits), _ptr(bi), _ptr(bv))
        return bi, bv, logits


class Reference:
    """The unmodified reference engine built from its sources (ref_harness.c)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (needs the reference sources)")
        L = C.CDLL(path)
        self.L = L
        for name in ("kqref_max_batch", "kqref_max_k", "kqref_pool_threads"):
            getattr(L, name).restype = C.c_int
        L.kqref_row_bytes.restype = C.c_uint64
        L.kqref_row_bytes.argtypes = [C.c_uint32, C.c_uint64]
        L.kqref_quantize_row_q8k.argtypes = [_vp, _vp, C.c_int]
        L.kqref_quantize_row_q8_0.argtypes = [_vp, _vp, C.c_int]
        L.kqref_dequant_row.argtypes = [C.c_uint32, _vp, C.c_int, _vp]
        L.kqref_load_input.restype = C.c_int
        L.kqref_load_input.argtypes = [_vp, _vp, C.c_int, C.c_int]
        L.kqref_row_batch.argtypes = [C.c_uint32, _vp, C.c_int, C.c_int, _vp]
        L.kqref_lm_row_dot.restype = C.c_float
        L.kqref_lm_row_dot.argtypes = [_vp, C.c_uint32, C.c_size_t, C.c_uint32, C.c_int, C.c_int]
        L.kqref_rmsnorm.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int]
        L.kqref_get_q8k.argtypes = [C.c_int, C.c_int, _vp]
        L.kqref_swiglu.argtypes = [_vp, _vp, C.c_int, C.c_int]
        L.kqref_turbo.argtypes = [C.c_int]
        L.kqref_dispatch.argtypes = [_vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int]
        L.kqref_dispatch_1thread.argtypes = [_vp, C.c_int, C.c_int, _vp, C.c_int]
        self.max_batch = L.kqref_max_batch()
        self.max_k = L.kqref_max_k()
        self.pool_threads = L.kqref_pool_threads()
        self._pool = False

    def init_pool(self):
        if not self._pool:
            self.L.kqref_init_pool()
            self._pool = True

    def quantize_q8k(self, x16):
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros((M, K // 256), dtype=Q8K_DTYPE)
        for m in range(M):
            self.L.kqref_quantize_row_q8k(_ptr(x16[m]), _ptr(out[m]), K)
        return out

    def quantize_q8_0(self, x16):
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros((M, K // 32), dtype=Q8_0_DTYPE)
        for m in range(M):
            self.L.kqref_quantize_row_q8_0(_ptr(x16[m]), _ptr(out[m]), K)
        return out

    def dequant(self, gtype, w, k):
        rows = w.shape[0]
        out = np.zeros((rows, k), dtype=np.float16)
        for r in range(rows):
            self.L.kqref_dequant_row(gtype, _ptr(np.ascontiguousarray(w[r])), k, _ptr(out[r]))
        return out

    def gemm(self, gtype, w, k, act):
        """The reference per-row batch kernels (sdot_row_<type>_batch) over all rows -> fp32 [M, rows]."""
        M = act.shape[0]
        act = np.ascontiguousarray(act)
        ok = self.L.kqref_load_input(None if gtype == TYPE_Q8_0 else _ptr(act),
                                     _ptr(act) if gtype == TYPE_Q8_0 else None, M, k)
        if not ok:
            raise ValueError(f"M={M}, K={k} exceed the reference input buffer")
        rows = w.shape[0]
        out = np.zeros((rows, M), dtype=np.float32)
        for r in range(rows):
            self.L.kqref_row_batch(gtype, _ptr(np.ascontiguousarray(w[r])), M, k, _ptr(out[r]))
        return np.ascontiguousarray(out.T)

    def lm_row_dot(self, gtype, w, k, act, row, m):
        act = np.ascontiguousarray(act)
        self.L.kqref_load_input(_ptr(act), None, act.shape[0], k)
        return np.float32(self.L.kqref_lm_row_dot(_ptr(np.ascontiguousarray(w)), gtype, w.shape[1], row, m, k))

    def rmsnorm(self, x16, gamma):
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros_like(x16)
        self.L.kqref_rmsnorm(_ptr(x16), _ptr(np.ascontiguousarray(gamma, dtype=np.float16)), _ptr(out), M, K)
        q = np.zeros((M, K // 256), dtype=Q8K_DTYPE)
        self.L.kqref_get_q8k(M, K, _ptr(q))
        return out, q

    def swiglu(self, gate, up):
        self.init_pool()
        g = np.array(gate, dtype=np.float16, copy=True, order="C")
        M, N = g.shape
        self.L.kqref_swiglu(_ptr(g), _ptr(np.ascontiguousarray(up, dtype=np.float16)), M, N)
        q = np.zeros((M, N // 256), dtype=Q8K_DTYPE)
        self.L.kqref_get_q8k(M, N, _ptr(q))
        return g, q

    class Task(C.Structure):
        _fields_ = [("w_base", C.c_void_p), ("type", C.c_uint32), ("rows", C.c_int),
                    ("dst", C.c_void_p), ("dst_stride", C.c_size_t),
                    ("residual", C.c_void_p), ("res_stride", C.c_size_t)]

    def dispatch(self, x16, tasks, prequantized=False):
        """sdot_gemm_multi_dispatch on the reference pool.  tasks: list of
        (gtype, w uint8[rows,row_bytes], dst fp16[M, stride], residual fp16[M, stride] or None)."""
        self.init_pool()
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        arr = (self.Task * len(tasks))()
        for i, (gtype, w, dst, res) in enumerate(tasks):
            arr[i].w_base = w.ctypes.data
            arr[i].type = gtype
            arr[i].rows = w.shape[0]
            arr[i].dst = dst.ctypes.data
            arr[i].dst_stride = dst.shape[1]
            arr[i].residual = None if res is None else res.ctypes.data
            arr[i].res_stride = 0 if res is None else res.shape[1]
        self.L.kqref_dispatch(_ptr(x16), M, K, C.cast(arr, C.c_void_p), len(tasks), int(bool(prequantized)))

    def dispatch_1thread(self, x16, tasks):
        """The same dispatch on the calling thread alone (the reference's job function over all rows)."""
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        arr = (self.Task * len(tasks))()
        for i, (gtype, w, dst, res) in enumerate(tasks):
            arr[i].w_base = w.ctypes.data
            arr[i].type = gtype
            arr[i].rows = w.shape[0]
            arr[i].dst = dst.ctypes.data
            arr[i].dst_stride = dst.shape[1]
            arr[i].residual = None if res is None else res.ctypes.data
            arr[i].res_stride = 0 if res is None else res.shape[1]
        self.L.kqref_dispatch_1thread(_ptr(x16), M, K, C.cast(arr, C.c_void_p), len(tasks))

    def turbo(self, on: bool):
        self.init_pool()
        self.L.kqref_turbo(1 if on else 0)

    class GgufTensor(C.Structure):
        _fields_ = [("name", C.c_char * 128), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4), ("type", C.c_uint32),
                    ("rel_offset", C.c_uint64), ("abs_offset", C.c_uint64), ("n_elems", C.c_uint64),
                    ("byte_size", C.c_uint64)]

    def gguf_parse(self, image: bytes):
        """parse_gguf_file (ENG:376-413) on a GGUF image: None if the reference rejects it, else
        (alignment, data_offset, [records as dicts])"""
        L = self.L
        L.kqref_gguf_parse.restype = C.c_int
        L.kqref_gguf_parse.argtypes = [C.c_char_p, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                       C.POINTER(C.c_uint64), _vp, C.c_int]
        recs = (self.GgufTensor * 512)()
        n, al, do = C.c_uint32(), C.c_uint64(), C.c_uint64()
        ok = L.kqref_gguf_parse(image, len(image), C.byref(n), C.byref(al), C.byref(do), C.cast(recs, C.c_void_p), 512)
        if ok != 1:
            return None
        out = [{"name": r.name.decode(), "n_dims": r.n_dims, "dims": list(r.dims), "type": r.type,
                "offset": r.abs_offset, "n_elems": r.n_elems, "bytes": r.byte_size} for r in recs[:n.value]]
        return al.value, do.value, out

    def gguf_find(self, image: bytes, name: str) -> int:
        """find_tensor (ENG:415-420): record index, -1 when absent, -2 when the image is rejected"""
        self.L.kqref_gguf_find.restype = C.c_int
        self.L.kqref_gguf_find.argtypes = [C.c_char_p, C.c_size_t, C.c_char_p]
        return self.L.kqref_gguf_find(image, len(image), name.encode())


def reference_available() -> bool:
    return os.path.exists(REF_SO)
