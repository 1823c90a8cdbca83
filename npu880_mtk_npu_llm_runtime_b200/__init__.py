"""B200 GGUF K-quant matmul path: Python front-end of libkq.so (include/kq.h).

The product is the C ABI in libkq.so (hand-written sm_100a CUDA kernels behind it).  This
module mirrors the reference engine's operator interface for the path
(src/v182_r22_breakthrough_engine.c: SdotMatrixTask ENG:888-899,
sdot_gemm_multi_dispatch ENG:4188, the per-row vec_dot kernels, the quantizers and producers)
over ctypes, for tests, benchmarks and Python callers.  Host arrays are numpy arrays; device
buffers are torch CUDA tensors (any object with data_ptr() works).

There is no CPU fallback: every compute call goes through libkq.so, and loading fails loudly
when the library is missing or no sm_100 device is present.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import synth  # noqa: F401  (re-exported helper)

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libkq.so")

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 0, 1, 8, 12, 13, 14
MAX_TASKS = 4

STATUS = {
    0: "KQ_OK", -1: "KQ_ERR_INVALID_ARGUMENT", -2: "KQ_ERR_UNSUPPORTED_TYPE", -3: "KQ_ERR_SHAPE",
    -4: "KQ_ERR_CUDA", -5: "KQ_ERR_OUT_OF_MEMORY", -6: "KQ_ERR_NO_DEVICE", -7: "KQ_ERR_TIMEOUT",
    -8: "KQ_ERR_NOT_READY", -9: "KQ_ERR_FORMAT", -10: "KQ_ERR_NOT_FOUND",
}

# BlockQ8K (ENG:868-872) / BlockQ8_0_Fast (ENG:874-877) as numpy records
Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsum32", "<i4", (8,))])
Q8_0_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (32,))])

# every symbol declared in include/*.h
EXPORTS = (
    "kq_version", "kq_status_string", "kq_init", "kq_destroy", "kq_set_stream", "kq_get_stream",
    "kq_synchronize", "kq_last_error", "kq_set_option", "kq_row_bytes",
    "kq_weight_upload", "kq_weight_upload_device", "kq_weight_free", "kq_weight_info",
    "kq_quantize_q8k", "kq_quantize_q8_0", "kq_quantize_q8k_async", "kq_quantize_q8_0_async",
    "kq_sdot_gemm_multi_dispatch", "kq_gemm_multi_async", "kq_gemm_multi_q8_async",
    "kq_sdot_row_batch", "kq_eval_single_lm_row_dot", "kq_debug_block_sums_async",
    "kq_rmsnorm_fp16_rows", "kq_swiglu_fp16_rows", "kq_rmsnorm_q8k_async", "kq_swiglu_q8k_async",
    "kq_run_ffn", "kq_run_ffn_async",
    "kq_lm_head_argmax", "kq_lm_head_argmax_async", "kq_lm_head_argmax_noalloc", "kq_eval_indexed_rows_argmax",
    "kq_dequant_rows", "kq_dequant_rows_async", "kq_embed_rows", "kq_embed_rows_async",
    "kq_gguf_open", "kq_gguf_open_memory", "kq_gguf_close", "kq_gguf_info", "kq_gguf_tensor_count",
    "kq_gguf_get_tensor", "kq_gguf_find_tensor", "kq_gguf_upload", "kq_gguf_upload_all",
    "kq_peer_region_bytes", "kq_peer_alloc", "kq_peer_free", "kq_peer_open", "kq_peer_close",
    "kq_gemm_peer_gather_async", "kq_peer_gather_wait_async",
    "kq_measure_int8_tops",
)

MAX_PEERS = 8
IPC_HANDLE_BYTES = 64


class PeerGatherStruct(C.Structure):
    """kq_peer_gather (include/kq.h): the ranks' gather regions of one sharded LM head."""
    _fields_ = [("world", C.c_int), ("rank", C.c_int), ("M", C.c_int), ("row_stride", C.c_longlong),
                ("row_begin", C.c_int), ("regions", C.c_void_p * 8)]


class GgufTensor(C.Structure):
    """kq_gguf_tensor: one record of a GGUF file's tensor directory (GgufTensorInfo, ENG:167-176)."""
    _fields_ = [("name", C.c_char_p), ("type", C.c_uint32), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("n_elems", C.c_uint64), ("offset", C.c_uint64), ("bytes", C.c_uint64), ("data", C.c_void_p)]


class KQError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class Task(C.Structure):
    """kq_task: one output matrix of a dispatch (mirrors SdotMatrixTask, ENG:888-899)."""
    _fields_ = [
        ("w", C.c_void_p), ("row_begin", C.c_int), ("rows", C.c_int),
        ("dst", C.c_void_p), ("dst_stride", C.c_size_t),
        ("residual", C.c_void_p), ("res_stride", C.c_size_t),
        ("dst_f32", C.c_void_p), ("dst_f32_stride", C.c_size_t),
    ]


_vp, _i, _u32, _sz, _u64 = C.c_void_p, C.c_int, C.c_uint32, C.c_size_t, C.c_uint64
_LIB = None


def load_library(path: str = LIB_PATH) -> C.CDLL:
    """Load libkq.so (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built: run `python -m npu880_mtk_npu_llm_runtime_b200.build`")
    L = C.CDLL(path)
    sig = {
        "kq_version": (C.c_char_p, []),
        "kq_status_string": (C.c_char_p, [_i]),
        "kq_init": (_i, [_i, C.POINTER(_vp)]),
        "kq_destroy": (_i, [_vp]),
        "kq_set_stream": (_i, [_vp, _vp]),
        "kq_get_stream": (_vp, [_vp]),
        "kq_synchronize": (_i, [_vp]),
        "kq_last_error": (C.c_char_p, [_vp]),
        "kq_set_option": (_i, [_vp, C.c_char_p, C.c_longlong]),
        "kq_row_bytes": (_u64, [_u32, _u64]),
        "kq_weight_upload": (_i, [_vp, _vp, _u32, _i, _i, C.POINTER(_vp)]),
        "kq_weight_upload_device": (_i, [_vp, _vp, _u32, _i, _i, C.POINTER(_vp)]),
        "kq_weight_free": (_i, [_vp, _vp]),
        "kq_weight_info": (_i, [_vp, C.POINTER(_u32), C.POINTER(_i), C.POINTER(_i), C.POINTER(_u64)]),
        "kq_quantize_q8k": (_i, [_vp, _vp, _i, _i, _vp]),
        "kq_quantize_q8_0": (_i, [_vp, _vp, _i, _i, _vp]),
        "kq_quantize_q8k_async": (_i, [_vp, _vp, _i, _i, _vp]),
        "kq_quantize_q8_0_async": (_i, [_vp, _vp, _i, _i, _vp]),
        "kq_sdot_gemm_multi_dispatch": (_i, [_vp, _vp, _i, _i, _vp, _i]),
        "kq_gemm_multi_async": (_i, [_vp, _vp, _sz, _i, _i, _vp, _i]),
        "kq_gemm_multi_q8_async": (_i, [_vp, _vp, _vp, _i, _i, _vp, _i]),
        "kq_sdot_row_batch": (_i, [_vp, _vp, _u32, _i, _vp]),
        "kq_eval_single_lm_row_dot": (_i, [_vp, _vp, _u32, _i, _vp]),
        "kq_debug_block_sums_async": (_i, [_vp, _vp, _i, _i, _vp, _i, _vp, _vp, _vp]),
        "kq_rmsnorm_fp16_rows": (_i, [_vp, _vp, _vp, _vp, _i, _i]),
        "kq_swiglu_fp16_rows": (_i, [_vp, _vp, _vp, _i, _i]),
        "kq_rmsnorm_q8k_async": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
        "kq_swiglu_q8k_async": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
        "kq_run_ffn": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
        "kq_run_ffn_async": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp, _vp]),
        "kq_lm_head_argmax": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp]),
        "kq_lm_head_argmax_async": (_i, [_vp, _vp, _vp, _i, _vp, _vp, _vp, _vp]),
        "kq_lm_head_argmax_noalloc": (_i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
        "kq_eval_indexed_rows_argmax": (_i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
        "kq_dequant_rows": (_i, [_vp, _vp, _i, _i, _vp]),
        "kq_dequant_rows_async": (_i, [_vp, _vp, _i, _i, _vp]),
        "kq_embed_rows": (_i, [_vp, _vp, _vp, _i, _vp]),
        "kq_embed_rows_async": (_i, [_vp, _vp, _vp, _i, _vp]),
        "kq_gguf_open": (_i, [C.c_char_p, C.POINTER(_vp)]),
        "kq_gguf_open_memory": (_i, [_vp, _sz, C.POINTER(_vp)]),
        "kq_gguf_close": (_i, [_vp]),
        "kq_gguf_info": (_i, [_vp, C.POINTER(_u32), C.POINTER(_u64), C.POINTER(_u64)]),
        "kq_gguf_tensor_count": (_i, [_vp]),
        "kq_gguf_get_tensor": (_i, [_vp, _i, C.POINTER(GgufTensor)]),
        "kq_gguf_find_tensor": (_i, [_vp, C.c_char_p]),
        "kq_gguf_upload": (_i, [_vp, _vp, _i, C.POINTER(_vp)]),
        "kq_gguf_upload_all": (_i, [_vp, _vp, C.POINTER(_vp), C.POINTER(_i)]),
        "kq_peer_region_bytes": (_sz, [_i, C.c_longlong]),
        "kq_peer_alloc": (_i, [_vp, _sz, C.POINTER(_vp), _vp]),
        "kq_peer_free": (_i, [_vp, _vp]),
        "kq_peer_open": (_i, [_vp, _vp, C.POINTER(_vp)]),
        "kq_peer_close": (_i, [_vp, _vp]),
        "kq_gemm_peer_gather_async": (_i, [_vp, _vp, _vp, C.POINTER(PeerGatherStruct), _vp]),
        "kq_peer_gather_wait_async": (_i, [_vp, C.POINTER(PeerGatherStruct), _vp]),
        "kq_measure_int8_tops": (_i, [_i, _i, C.POINTER(C.c_double)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _LIB = L
    return L


def row_bytes(gtype: int, k: int) -> int:
    return int(load_library().kq_row_bytes(gtype, k))


def _hp(a):
    """host pointer of a numpy array (C-contiguous) or None"""
    if a is None:
        return None
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("host arrays must be C-contiguous")
    return a.ctypes.data


def _dp(t):
    """device pointer of a torch CUDA tensor (or any object with data_ptr()), or None"""
    if t is None:
        return None
    return t.data_ptr()


class Weight:
    """A GGUF tensor resident in HBM (kq_weight)."""

    def __init__(self, ctx: "Context", handle: int, gtype: int, rows: int, cols: int):
        self.ctx, self.handle, self.type, self.rows, self.cols = ctx, handle, gtype, rows, cols

    @property
    def device_bytes(self) -> int:
        b = C.c_uint64()
        self.ctx.L.kq_weight_info(self.handle, None, None, None, C.byref(b))
        return b.value

    def free(self):
        if self.handle:
            self.ctx.L.kq_weight_free(self.ctx.handle, self.handle)
            self.handle = None


class Context:
    """kq_ctx: one CUDA device and stream (replaces the engine's pinned pool, ENG:3843)."""

    def __init__(self, device: int = 0):
        self.L = load_library()
        h = _vp()
        st = self.L.kq_init(device, C.byref(h))
        if st != 0:
            raise KQError(st, f"kq_init(device={device}) failed (an sm_100 CUDA device is required)")
        self.handle = h.value
        self.device = device

    # ---- plumbing
    def check(self, st: int):
        if st != 0:
            raise KQError(st, self.L.kq_last_error(self.handle).decode())

    def close(self):
        if self.handle:
            self.L.kq_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def set_stream(self, stream_ptr: int):
        self.check(self.L.kq_set_stream(self.handle, stream_ptr))

    @property
    def stream(self) -> int:
        return self.L.kq_get_stream(self.handle) or 0

    def synchronize(self):
        self.check(self.L.kq_synchronize(self.handle))

    def set_option(self, name: str, value: int):
        self.check(self.L.kq_set_option(self.handle, name.encode(), int(value)))

    # ---- weights
    def upload(self, gguf: np.ndarray, gtype: int, rows: int, cols: int) -> Weight:
        h = _vp()
        self.check(self.L.kq_weight_upload(self.handle, _hp(np.ascontiguousarray(gguf)), gtype, rows, cols, C.byref(h)))
        return Weight(self, h.value, gtype, rows, cols)

    def upload_device(self, gguf_dev, gtype: int, rows: int, cols: int) -> Weight:
        h = _vp()
        self.check(self.L.kq_weight_upload_device(self.handle, _dp(gguf_dev), gtype, rows, cols, C.byref(h)))
        return Weight(self, h.value, gtype, rows, cols)

    # ---- host-pointer (drop-in, blocking) entry points
    def quantize_q8k(self, x16: np.ndarray) -> np.ndarray:
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros((M, K // 256), dtype=Q8K_DTYPE)
        self.check(self.L.kq_quantize_q8k(self.handle, _hp(x16), M, K, _hp(out)))
        return out

    def quantize_q8_0(self, x16: np.ndarray) -> np.ndarray:
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros((M, K // 32), dtype=Q8_0_DTYPE)
        self.check(self.L.kq_quantize_q8_0(self.handle, _hp(x16), M, K, _hp(out)))
        return out

    def sdot_gemm_multi_dispatch(self, x16: np.ndarray, tasks):
        """sdot_gemm_multi_dispatch (ENG:4188) with host arrays.  tasks: list of dicts with keys
        w (Weight), dst (fp16 [M, stride] or None), residual (fp16 or None), dst_f32 (fp32 or None),
        row_begin (default 0), rows (default w.rows), or an array made once by make_host_tasks for
        calls that repeat.  Outputs are written in place."""
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        arr = tasks if isinstance(tasks, C.Array) else self.make_host_tasks(tasks)
        self.check(self.L.kq_sdot_gemm_multi_dispatch(self.handle, _hp(x16), M, K, arr, len(arr)))

    @staticmethod
    def make_host_tasks(tasks):
        """kq_task array over HOST arrays (the arrays must outlive every call that uses it)"""
        arr = (Task * len(tasks))()
        for i, t in enumerate(tasks):
            w = t["w"]
            arr[i].w = w.handle
            arr[i].row_begin = t.get("row_begin", 0)
            arr[i].rows = t.get("rows", w.rows - arr[i].row_begin)
            for key, skey in (("dst", "dst_stride"), ("residual", "res_stride"), ("dst_f32", "dst_f32_stride")):
                a = t.get(key)
                if a is not None:
                    setattr(arr[i], key, _hp(a))
                    setattr(arr[i], skey, a.shape[1])
        return arr

    def sdot_row_batch(self, w: Weight, row: int, M: int) -> np.ndarray:
        out = np.zeros(M, dtype=np.float32)
        self.check(self.L.kq_sdot_row_batch(self.handle, w.handle, row, M, _hp(out)))
        return out

    def eval_single_lm_row_dot(self, w: Weight, row: int, m: int) -> np.float32:
        out = np.zeros(1, dtype=np.float32)
        self.check(self.L.kq_eval_single_lm_row_dot(self.handle, w.handle, row, m, _hp(out)))
        return out[0]

    def rmsnorm_fp16_rows(self, x16: np.ndarray, gamma: np.ndarray) -> np.ndarray:
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M, K = x16.shape
        out = np.zeros_like(x16)
        self.check(self.L.kq_rmsnorm_fp16_rows(self.handle, _hp(x16), _hp(np.ascontiguousarray(gamma, np.float16)),
                                               _hp(out), M, K))
        return out

    def swiglu_fp16_rows(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        g = np.array(gate, dtype=np.float16, copy=True, order="C")
        M, N = g.shape
        self.check(self.L.kq_swiglu_fp16_rows(self.handle, _hp(g), _hp(np.ascontiguousarray(up, np.float16)), M, N))
        return g

    def run_ffn(self, gate: Weight, up: Weight, down: Weight, x16: np.ndarray, gamma: np.ndarray) -> np.ndarray:
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        out = np.zeros_like(x16)
        self.check(self.L.kq_run_ffn(self.handle, gate.handle, up.handle, down.handle, x16.shape[0], _hp(x16),
                                     _hp(np.ascontiguousarray(gamma, np.float16)), _hp(out)))
        return out

    def lm_head_argmax(self, w: Weight, x16: np.ndarray, want_logits: bool = True):
        x16 = np.ascontiguousarray(x16, dtype=np.float16)
        M = x16.shape[0]
        logits = np.zeros((M, w.rows), dtype=np.float16) if want_logits else None
        toks = np.zeros(M, dtype=np.uint32)
        vals = np.zeros(M, dtype=np.float32)
        self.check(self.L.kq_lm_head_argmax(self.handle, w.handle, _hp(x16), M, _hp(logits), _hp(toks), _hp(vals)))
        return toks, vals, logits

    def eval_indexed_rows_argmax(self, w: Weight, row_ids: np.ndarray, M: int, top_toks=None, top_vals=None,
                                 logits_m1=None):
        ids = np.ascontiguousarray(row_ids, dtype=np.uint32)
        toks = np.zeros(M, np.uint32) if top_toks is None else top_toks
        vals = np.full(M, -1e30, np.float32) if top_vals is None else top_vals
        self.check(self.L.kq_eval_indexed_rows_argmax(self.handle, w.handle, _hp(ids), ids.shape[0], M,
                                                      _hp(logits_m1), _hp(toks), _hp(vals)))
        return toks, vals

    def dequant_rows(self, w: Weight, row_begin: int = 0, rows: int | None = None) -> np.ndarray:
        rows = w.rows - row_begin if rows is None else rows
        out = np.zeros((rows, w.cols), dtype=np.float16)
        self.check(self.L.kq_dequant_rows(self.handle, w.handle, row_begin, rows, _hp(out)))
        return out

    def embed_rows(self, w: Weight, ids) -> np.ndarray:
        """fp16 rows ids[i] of w (the embedding lookup of ENG:8667-8670)"""
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros((len(ids), w.cols), dtype=np.float16)
        self.check(self.L.kq_embed_rows(self.handle, w.handle, _hp(ids), len(ids), _hp(out)))
        return out

    def embed_rows_async(self, w: Weight, ids_dev, n: int, out_dev):
        self.check(self.L.kq_embed_rows_async(self.handle, w.handle, _dp(ids_dev), n, _dp(out_dev)))

    # ---- device-pointer (async) entry points
    @staticmethod
    def make_tasks(tasks):
        arr = (Task * len(tasks))()
        for i, t in enumerate(tasks):
            w = t["w"]
            arr[i].w = w.handle
            arr[i].row_begin = t.get("row_begin", 0)
            arr[i].rows = t.get("rows", w.rows - arr[i].row_begin)
            for key, skey in (("dst", "dst_stride"), ("residual", "res_stride"), ("dst_f32", "dst_f32_stride")):
                a = t.get(key)
                if a is not None:
                    setattr(arr[i], key, _dp(a))
                    setattr(arr[i], skey, t.get(skey, a.shape[-1]))
        return arr

    def gemm_multi_async(self, x_dev, M: int, K: int, tasks, x_stride: int | None = None):
        arr = tasks if isinstance(tasks, C.Array) else self.make_tasks(tasks)
        self.check(self.L.kq_gemm_multi_async(self.handle, _dp(x_dev), x_stride or K, M, K, arr, len(arr)))

    def gemm_multi_q8_async(self, act_q8k_dev, act_q80_dev, M: int, K: int, tasks):
        arr = tasks if isinstance(tasks, C.Array) else self.make_tasks(tasks)
        self.check(self.L.kq_gemm_multi_q8_async(self.handle, _dp(act_q8k_dev), _dp(act_q80_dev), M, K, arr, len(arr)))

    def quantize_q8k_async(self, x_dev, M: int, K: int, out_dev):
        self.check(self.L.kq_quantize_q8k_async(self.handle, _dp(x_dev), M, K, _dp(out_dev)))

    def quantize_q8_0_async(self, x_dev, M: int, K: int, out_dev):
        self.check(self.L.kq_quantize_q8_0_async(self.handle, _dp(x_dev), M, K, _dp(out_dev)))

    def debug_block_sums_async(self, w: Weight, row_begin: int, rows: int, act_dev, M: int, sumi_dev, summ_dev,
                               out_f32_dev=None):
        self.check(self.L.kq_debug_block_sums_async(self.handle, w.handle, row_begin, rows, _dp(act_dev), M,
                                                    _dp(sumi_dev), _dp(summ_dev), _dp(out_f32_dev)))

    def rmsnorm_q8k_async(self, x_dev, gamma_dev, out_dev, M: int, K: int, q8k_dev=None):
        self.check(self.L.kq_rmsnorm_q8k_async(self.handle, _dp(x_dev), _dp(gamma_dev), _dp(out_dev), M, K,
                                               _dp(q8k_dev)))

    def swiglu_q8k_async(self, gate_dev, up_dev, M: int, N: int, q8k_dev=None):
        self.check(self.L.kq_swiglu_q8k_async(self.handle, _dp(gate_dev), _dp(up_dev), M, N, _dp(q8k_dev)))

    def run_ffn_async(self, gate: Weight, up: Weight, down: Weight, M: int, x_dev, gamma_dev, out_dev):
        self.check(self.L.kq_run_ffn_async(self.handle, gate.handle, up.handle, down.handle, M, _dp(x_dev),
                                           _dp(gamma_dev), _dp(out_dev)))

    # ---- several GPUs: the gather in the LM head GEMV (kq_peer_*, kq_gemm_peer_gather_async)
    def peer_region_bytes(self, M: int, row_stride: int) -> int:
        return int(self.L.kq_peer_region_bytes(M, row_stride))

    def peer_alloc(self, nbytes: int):
        """(device pointer, IPC handle bytes) of a zeroed gather region on this context's device"""
        ptr = _vp()
        h = (C.c_ubyte * IPC_HANDLE_BYTES)()
        self.check(self.L.kq_peer_alloc(self.handle, nbytes, C.byref(ptr), h))
        return int(ptr.value), bytes(h)

    def peer_free(self, ptr: int):
        self.check(self.L.kq_peer_free(self.handle, ptr))

    def peer_open(self, handle: bytes) -> int:
        ptr = _vp()
        buf = (C.c_ubyte * IPC_HANDLE_BYTES).from_buffer_copy(handle)
        self.check(self.L.kq_peer_open(self.handle, buf, C.byref(ptr)))
        return int(ptr.value)

    def peer_close(self, ptr: int):
        self.check(self.L.kq_peer_close(self.handle, ptr))

    def gemm_peer_gather_async(self, w: Weight, x_dev, pg: PeerGatherStruct, out_dev=None):
        self.check(self.L.kq_gemm_peer_gather_async(self.handle, w.handle, _dp(x_dev), C.byref(pg), _dp(out_dev)))

    def peer_gather_wait_async(self, pg: PeerGatherStruct, out_dev=None):
        self.check(self.L.kq_peer_gather_wait_async(self.handle, C.byref(pg), _dp(out_dev)))

    def lm_head_argmax_async(self, w: Weight, x_dev, M: int, logits_dev=None, logits_f32_dev=None, toks_dev=None,
                             vals_dev=None):
        self.check(self.L.kq_lm_head_argmax_async(self.handle, w.handle, _dp(x_dev), M, _dp(logits_dev),
                                                  _dp(logits_f32_dev), _dp(toks_dev), _dp(vals_dev)))

    def dequant_rows_async(self, w: Weight, row_begin: int, rows: int, out_dev):
        self.check(self.L.kq_dequant_rows_async(self.handle, w.handle, row_begin, rows, _dp(out_dev)))


def q8k_bytes(M: int, K: int) -> int:
    return M * (K // 256) * 292


def q8_0_bytes(M: int, K: int) -> int:
    return M * (K // 32) * 36


class Gguf:
    """A GGUF v2/v3 file's tensor directory (kq_gguf): from a path (mapped read-only) or from bytes
    in memory (kept alive by this object).  Mirrors parse_gguf_file / find_tensor (ENG:376-420)."""

    def __init__(self, path: str | None = None, data: bytes | np.ndarray | None = None):
        self.L = load_library()
        h = _vp()
        self._buf = None
        if path is not None:
            st = self.L.kq_gguf_open(path.encode(), C.byref(h))
        else:
            self._buf = np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray)) else np.ascontiguousarray(data)
            st = self.L.kq_gguf_open_memory(_hp(self._buf), self._buf.nbytes, C.byref(h))
        if st != 0:
            raise KQError(st, f"kq_gguf_open: {STATUS.get(st, st)}")
        self.handle = h.value

    def close(self):
        if self.handle:
            self.L.kq_gguf_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def info(self):
        v, a, d = C.c_uint32(), C.c_uint64(), C.c_uint64()
        self.L.kq_gguf_info(self.handle, C.byref(v), C.byref(a), C.byref(d))
        return {"version": v.value, "alignment": a.value, "data_offset": d.value}

    def __len__(self) -> int:
        return self.L.kq_gguf_tensor_count(self.handle)

    def tensor(self, index: int) -> dict:
        t = GgufTensor()
        st = self.L.kq_gguf_get_tensor(self.handle, index, C.byref(t))
        if st != 0:
            raise KQError(st, f"tensor {index}")
        return {"name": t.name.decode(), "type": t.type, "n_dims": t.n_dims, "dims": list(t.dims),
                "n_elems": t.n_elems, "offset": t.offset, "bytes": t.bytes, "data": t.data}

    def find(self, name: str) -> int:
        return self.L.kq_gguf_find_tensor(self.handle, name.encode())

    def upload(self, ctx: "Context", index: int) -> Weight:
        h = _vp()
        ctx.check(self.L.kq_gguf_upload(ctx.handle, self.handle, index, C.byref(h)))
        t = self.tensor(index)
        return Weight(ctx, h.value, t["type"], t["dims"][1], t["dims"][0])

    def upload_all(self, ctx: "Context") -> list:
        """one Weight per quantized matrix of the file, None for the other records"""
        n = len(self)
        arr = (_vp * max(1, n))()
        cnt = _i()
        ctx.check(self.L.kq_gguf_upload_all(ctx.handle, self.handle, arr, C.byref(cnt)))
        out = []
        for i in range(n):
            if arr[i]:
                t = self.tensor(i)
                out.append(Weight(ctx, arr[i], t["type"], t["dims"][1], t["dims"][0]))
            else:
                out.append(None)
        return out
