"""Seeded synthetic GGUF weight rows and activations for the K-quant matmul path.

The byte layouts are the GGUF block formats the reference engine reads straight from its
mmap (src/v182_r22_breakthrough_engine.c):

* Q4_K, 144 B per 256 values: fp16 d, fp16 dmin, 12 packed scale/min bytes, 128 nibble bytes
  (dequant_block_q4_k, ENG:758-801; get_scale_min_k4, ENG:743-749).
* Q5_K, 176 B per 256: d, dmin, 12 scale bytes, qh[32], qs[128] (ENG:803-853).
* Q6_K, 210 B per 256: ql[128], qh[64], int8 scales[16], fp16 d at byte 208 (ENG:673-741).
* Q8_0, 34 B per 32: fp16 d, int8 qs[32] (ENG:598-615).

Value distributions follow the benchmark configurations: nibbles / 5-bit / 6-bit quants
uniform over their range, Q4_K/Q5_K sub-block scales and mins uniform 0..63, Q6_K scales
uniform -32..31, Q8_0 quants uniform -127..127, and every fp16 block scale |N(0, 1e-3)|.
Activations are fp32 N(0, 1) rounded to fp16, the engine's activation type.
"""
from __future__ import annotations

import numpy as np

TYPE_F32 = 0
TYPE_F16 = 1
TYPE_Q8_0 = 8
TYPE_Q4_K = 12
TYPE_Q5_K = 13
TYPE_Q6_K = 14

TYPE_NAMES = {TYPE_Q8_0: "q8_0", TYPE_Q4_K: "q4_k", TYPE_Q5_K: "q5_k", TYPE_Q6_K: "q6_k"}
BLOCK_ELEMS = {TYPE_Q8_0: 32, TYPE_Q4_K: 256, TYPE_Q5_K: 256, TYPE_Q6_K: 256}
BLOCK_BYTES = {TYPE_Q8_0: 34, TYPE_Q4_K: 144, TYPE_Q5_K: 176, TYPE_Q6_K: 210}


def row_bytes(gtype: int, k: int) -> int:
    """compute_ggml_bytes (ENG:364-374) for one row of k values."""
    if gtype == TYPE_F32:
        return 4 * k
    if gtype == TYPE_F16:
        return 2 * k
    return (k // BLOCK_ELEMS[gtype]) * BLOCK_BYTES[gtype]


def _scale_f16(rng: np.random.Generator, n: int) -> np.ndarray:
    return np.abs(rng.normal(0.0, 1e-3, size=n)).astype(np.float16).view(np.uint8).reshape(n, 2)


def _int8_draw(rng: np.random.Generator, span: tuple[int, int], shape) -> np.ndarray:
    """int8 values uniform in [lo, hi) as bytes (hi <= 128)."""
    return rng.integers(span[0], span[1], size=shape, dtype=np.int8).view(np.uint8)


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of get_scale_min_k4 (ENG:743-749): pack eight 6-bit scales and eight 6-bit mins
    per super-block into 12 bytes.  sc, mn: uint8 [..., 8] with values 0..63."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros(sc.shape[:-1] + (12,), dtype=np.uint8)
    # sub-blocks 0..3: 6 bits in bytes 0..3 (scale) and 4..7 (min)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    # sub-blocks 4..7: low nibbles in bytes 8..11, top two bits in the spare bits above
    out[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((mn[..., 4:8] & 0x0F) << 4)
    return out


def gen_weights(gtype: int, rows: int, k: int, seed: int, q6_scales: tuple[int, int] = (-32, 32),
                q8_quants: tuple[int, int] = (-127, 128)) -> np.ndarray:
    """rows x k weights of GGUF type gtype as raw row-major block bytes: uint8[rows, row_bytes].
    q6_scales / q8_quants: [lo, hi) of the Q6_K sub-block scales and the Q8_0 quants; the
    defaults are the benchmark distributions, (-128, 128) covers every value a GGUF file can hold
    (the reference's Q6_K quantizer maps each block's largest scale to -128)."""
    if k % BLOCK_ELEMS[gtype]:
        raise ValueError(f"k={k} is not a multiple of the {TYPE_NAMES[gtype]} block size")
    rng = np.random.default_rng(seed)
    nb = rows * (k // BLOCK_ELEMS[gtype])
    blk = np.empty((nb, BLOCK_BYTES[gtype]), dtype=np.uint8)
    if gtype in (TYPE_Q4_K, TYPE_Q5_K):
        blk[:, 0:2] = _scale_f16(rng, nb)
        blk[:, 2:4] = _scale_f16(rng, nb)
        sc = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, size=(nb, 8), dtype=np.uint8)
        blk[:, 4:16] = pack_scale_min_k4(sc, mn)
        if gtype == TYPE_Q4_K:
            blk[:, 16:144] = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
        else:
            blk[:, 16:176] = rng.integers(0, 256, size=(nb, 160), dtype=np.uint8)
    elif gtype == TYPE_Q6_K:
        blk[:, 0:192] = rng.integers(0, 256, size=(nb, 192), dtype=np.uint8)
        blk[:, 192:208] = _int8_draw(rng, q6_scales, (nb, 16))
        blk[:, 208:210] = _scale_f16(rng, nb)
    elif gtype == TYPE_Q8_0:
        blk[:, 0:2] = _scale_f16(rng, nb)
        blk[:, 2:34] = _int8_draw(rng, q8_quants, (nb, 32))
    else:
        raise ValueError(f"unsupported type {gtype}")
    return blk.reshape(rows, row_bytes(gtype, k))


def gen_activations(m: int, k: int, seed: int) -> np.ndarray:
    """fp32 N(0, 1) activations rounded to fp16 (the engine's activation type): float16[m, k]."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(size=(m, k), dtype=np.float32).astype(np.float16)


def gen_gamma(k: int, seed: int) -> np.ndarray:
    """RMSNorm weights around 1.0 as fp16."""
    rng = np.random.default_rng(seed)
    return (1.0 + 0.1 * rng.standard_normal(size=k)).astype(np.float16)


# ---------------------------------------------------------------- GGUF files

GGUF_U32, GGUF_F32, GGUF_STRING, GGUF_ARRAY, GGUF_U64 = 4, 6, 8, 9, 10


def write_gguf(tensors, kv=None, version: int = 3, alignment: int | None = None) -> bytes:
    """A GGUF v2/v3 image (the file format the engine mmaps, parsed by ENG:376-413): header, the
    key/value pairs `kv` ([(key, value_type, value)]; value_type GGUF_U32 / GGUF_U64 / GGUF_F32 /
    GGUF_STRING, or (GGUF_ARRAY, element type) with a list), the tensor records of `tensors`
    ([(name, ggml_type, dims, data_bytes)], dims[0] = values per row) and the data section, each
    tensor at a multiple of the alignment (general.alignment when given, else 32)."""
    import struct

    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    def scalar(t, v) -> bytes:
        return {GGUF_U32: lambda: struct.pack("<I", v), GGUF_U64: lambda: struct.pack("<Q", v),
                GGUF_F32: lambda: struct.pack("<f", v), GGUF_STRING: lambda: s(v)}[t]()

    kv = list(kv or [])
    if alignment is not None:
        kv.append(("general.alignment", GGUF_U32, alignment))
    align = alignment or 32
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv)))
    for key, t, v in kv:
        out += s(key)
        if isinstance(t, tuple):
            out += struct.pack("<IIQ", GGUF_ARRAY, t[1], len(v)) + b"".join(scalar(t[1], e) for e in v)
        else:
            out += struct.pack("<I", t) + scalar(t, v)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off = (off + len(data) + align - 1) // align * align
    for (name, gtype, dims, _), o in zip(tensors, offsets):
        out += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gtype, o)
    out += bytes((-len(out)) % align)
    base = len(out)
    for (_, _, _, data), o in zip(tensors, offsets):
        out += bytes(base + o - len(out)) + bytes(data)
    return bytes(out)
