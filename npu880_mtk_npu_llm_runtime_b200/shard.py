"""Vocabulary sharding of the LM head over ranks (one process per GPU).

The reference scans the whole vocabulary on one device (run_final_norm_and_lm_head_pipelined,
src/v182_r22_breakthrough_engine.c:9686-9707: fp16 logits of each 24832-row chunk, then the
first maximal row, strict '>').  Split over N ranks, rank r owns rows [r * C, min(V, (r+1) * C))
with C = ceil(V / N); each rank reduces its slice to one (value, row) pair per activation row and
the pairs are exchanged with one all-gather.  merge_argmax picks, per activation row, the largest
value and among equal values the smallest row -- the reference's first-maximal-row rule applied
to the concatenated slices.
"""
from __future__ import annotations

import numpy as np


def vocab_slice(rank: int, world: int, vocab: int) -> tuple[int, int]:
    """(first row, rows) of this rank's vocabulary slice."""
    chunk = (vocab + world - 1) // world
    first = rank * chunk
    return first, max(0, min(vocab, first + chunk) - first)


def merge_argmax(vals: np.ndarray, rows: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """vals, rows: [world, M] per-rank maxima and their global rows (rows < 0: empty slice).
    Returns the per-column (row, value) of the largest value, smallest row on ties."""
    vals = np.asarray(vals, dtype=np.float32)
    rows = np.asarray(rows, dtype=np.int64)
    world, M = vals.shape
    best_v = np.full(M, -np.inf, dtype=np.float32)
    best_r = np.full(M, -1, dtype=np.int64)
    for r in range(world):
        v, i = vals[r], rows[r]
        ok = i >= 0
        take = ok & ((v > best_v) | ((v == best_v) & ((best_r < 0) | (i < best_r))))
        best_v = np.where(take, v, best_v)
        best_r = np.where(take, i, best_r)
    return best_r, best_v


def gather_argmax_torch(vals, rows, group=None):
    """All-gather per-rank (value, global row) pairs with torch.distributed and merge them.
    vals: float32 [M], rows: int64 [M] tensors on this rank's device; returns numpy (rows, vals)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    pair = torch.stack([vals.float(), rows.double().float()], dim=0)  # rows < 2^24: exact in fp32
    out = torch.zeros((world * pair.shape[0], pair.shape[1]), dtype=pair.dtype, device=pair.device)
    dist.all_gather_into_tensor(out, pair, group=group)
    o = out.cpu().numpy().reshape(world, 2, -1)
    return merge_argmax(o[:, 0, :], o[:, 1, :].astype(np.int64))
