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

import ctypes as C

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


# ---------------------------------------------------------------------------- FFN row sharding

def balanced_split(n: int, world: int) -> list[tuple[int, int]]:
    """(first, count) of each rank's contiguous share of n items; the first n % world ranks take
    one more."""
    q, r = divmod(n, world)
    out, first = [], 0
    for k in range(world):
        c = q + (1 if k < r else 0)
        out.append((first, c))
        first += c
    return out


class FfnShardPlan:
    """Row sharding of the FFN block x_out = x + W_down . swiglu(W_gate . xn, W_up . xn),
    xn = rmsnorm(x) (the engine's SDOT FFN sequence, src/v182_r22_breakthrough_engine.c:8283-8298),
    over `world` ranks, one process per GPU:

      * rank r owns intermediate values [inter_first, inter_first + inter_count) in whole
        256-value blocks -- those rows of W_gate and W_up, so its SwiGLU inputs are local -- and
        quantizes its slice of the SwiGLU output to Q8_K itself: Q8_K blocks are independent
        (one scale per 256 values), so the slices concatenate to the full row's Q8_K;
      * one all-gather of the Q8_K blocks (292 bytes per 256 values, every rank padded to the
        largest share) gives every rank the whole intermediate activation;
      * rank r owns hidden rows [hid_first, hid_first + hid_count) of W_down in whole 16-row
        groups (the device tile height) and writes that slice of x_out (residual added), and a
        second all-gather assembles x_out.

    Every output value is computed by exactly the operations of the unsharded block, so the
    sharded result is bit-identical to it."""

    def __init__(self, hidden: int, ffn: int, world: int):
        if hidden % 256 or ffn % 256:
            raise ValueError("hidden and ffn must be multiples of 256")
        self.hidden, self.ffn, self.world = hidden, ffn, world
        self.inter_blocks = [(f, c) for f, c in balanced_split(ffn // 256, world)]
        self.hid_groups = [(f, c) for f, c in balanced_split(hidden // 16, world)]
        self.inter_max = max(c for _, c in self.inter_blocks)        # blocks per rank, padded
        self.hid_max = max(c for _, c in self.hid_groups) * 16       # hidden rows per rank, padded

    def inter(self, rank: int) -> tuple[int, int]:
        """(first value, values) of rank's intermediate slice"""
        f, c = self.inter_blocks[rank]
        return f * 256, c * 256

    def hid(self, rank: int) -> tuple[int, int]:
        """(first row, rows) of rank's hidden slice of W_down / x_out"""
        f, c = self.hid_groups[rank]
        return f * 16, c * 16

    def inter_index(self) -> np.ndarray:
        """positions, in the gathered [world * inter_max] block axis, of blocks 0 .. ffn/256 - 1"""
        return np.concatenate([r * self.inter_max + np.arange(c) for r, (_, c) in enumerate(self.inter_blocks)])

    def hid_index(self) -> np.ndarray:
        """positions, in the gathered [world * hid_max] column axis, of hidden columns 0 .. hidden - 1"""
        return np.concatenate([r * self.hid_max + np.arange(c * 16) for r, (_, c) in enumerate(self.hid_groups)])


class RowShardedFfn:
    """One rank's part of the row-sharded FFN block on its GPU (plan: FfnShardPlan).  The rank holds
    its rows of W_gate / W_up / W_down (kq Weight objects of plan.inter(rank)[1] / plan.hid(rank)[1]
    rows) and preallocated buffers, so a step allocates nothing and can be captured in a CUDA graph
    together with the collectives.  A step (forward):

      1. RMSNorm + Q8_K of the whole input rows (every rank);
      2. its gate / up rows (one dispatch, two tasks) -> fp16 [M, C];
      3. SwiGLU + Q8_K of its slice -> send buffer of M * inter_max Q8_K blocks;
      4. all-gather of the send buffers, then the Q8_K blocks put in row order (one index_select);
      5. its rows of W_down with the residual -> fp16 send buffer [M, hid_max];
      6. all-gather, then the output columns put in row order into y.

    all_gather(out, inp) is torch.distributed.all_gather_into_tensor (NCCL) on real ranks; a test
    may pass a function that emulates it.  Everything -- the library calls, the index gathers and
    the collectives -- is ordered on the context's CUDA stream."""

    def __init__(self, ctx, plan: FfnShardPlan, rank: int, M: int, device):
        import torch
        self.ctx, self.plan, self.rank, self.M = ctx, plan, rank, M
        hid, ffn, W = plan.hidden, plan.ffn, plan.world
        self.c0, self.C = plan.inter(rank)
        self.r0, self.R = plan.hid(rank)
        u8, f16 = torch.uint8, torch.float16
        self.xn = torch.empty((M, hid), dtype=f16, device=device)
        self.q_x = torch.empty((M * (hid // 256) * 292,), dtype=u8, device=device)
        self.g = torch.empty((M, self.C), dtype=f16, device=device)
        self.u = torch.empty((M, self.C), dtype=f16, device=device)
        self.h_send = torch.zeros((M * plan.inter_max * 292,), dtype=u8, device=device)
        self.h_all = torch.zeros((W * M * plan.inter_max * 292,), dtype=u8, device=device)
        self.h_full = torch.empty((M * (ffn // 256) * 292,), dtype=u8, device=device)
        self.o_send = torch.zeros((M, plan.hid_max), dtype=f16, device=device)
        self.o_all = torch.zeros((W * M * plan.hid_max,), dtype=f16, device=device)
        # block (m, j) of the intermediate: rank r's send buffer holds its blocks row-major
        # [M][count_r] from offset 0 (SwiGLU writes its Q8_K rows contiguously)
        idx = np.empty((M, ffn // 256), np.int64)
        for r, (first, cnt) in enumerate(plan.inter_blocks):
            for m in range(M):
                idx[m, first:first + cnt] = r * M * plan.inter_max + m * cnt + np.arange(cnt)
        self.h_idx = torch.from_numpy(idx.reshape(-1)).to(device)
        # column c of output row m: rank r's send buffer is [M][hid_max] with its rows first
        oidx = np.empty((M, hid), np.int64)
        for r, (first, cnt) in enumerate(plan.hid_groups):
            for m in range(M):
                oidx[m, first * 16:(first + cnt) * 16] = (r * M + m) * plan.hid_max + np.arange(cnt * 16)
        self.o_idx = torch.from_numpy(oidx.reshape(-1)).to(device)

    def tasks(self, gate, up, down, x):
        """kq task arrays of one weight set (its row slices) for input/residual x [M, hidden]"""
        ctx = self.ctx
        gu = ctx.make_tasks([dict(w=gate, dst=self.g, dst_stride=self.C), dict(w=up, dst=self.u, dst_stride=self.C)])
        dn = ctx.make_tasks([dict(w=down, dst=self.o_send, dst_stride=self.plan.hid_max,
                                  residual=x[:, self.r0:], res_stride=self.plan.hidden)])
        return gu, dn

    def part1(self, x, gamma, gu_tasks):
        M, hid, ctx = self.M, self.plan.hidden, self.ctx
        ctx.rmsnorm_q8k_async(x, gamma, self.xn, M, hid, self.q_x)
        ctx.gemm_multi_q8_async(self.q_x, None, M, hid, gu_tasks)
        ctx.swiglu_q8k_async(self.g, self.u, M, self.C, self.h_send)

    def _on_ctx_stream(self):
        import torch
        return torch.cuda.stream(torch.cuda.ExternalStream(self.ctx.stream, device=self.h_idx.device))

    def assemble_inter(self):
        import torch
        with self._on_ctx_stream():
            torch.index_select(self.h_all.view(-1, 292), 0, self.h_idx, out=self.h_full.view(-1, 292))

    def part2(self, dn_tasks):
        self.ctx.gemm_multi_q8_async(self.h_full, None, self.M, self.plan.ffn, dn_tasks)

    def assemble_out(self, y):
        import torch
        with self._on_ctx_stream():
            torch.index_select(self.o_all, 0, self.o_idx, out=y.view(-1))

    def forward(self, x, gamma, y, gu_tasks, dn_tasks, all_gather):
        self.part1(x, gamma, gu_tasks)
        with self._on_ctx_stream():
            all_gather(self.h_all, self.h_send)
        self.assemble_inter()
        self.part2(dn_tasks)
        with self._on_ctx_stream():
            all_gather(self.o_all, self.o_send.view(-1))
        self.assemble_out(y)


class PeerGather:
    """The vocabulary-sharded LM head with its all-gather inside the GEMV (kq_peer_gather).

    Each rank owns a region (two buffers of [M][vocab] tagged 64-bit entries and control words);
    the regions are exchanged as IPC handles and opened by every rank.  gather(w, x) runs this
    rank's slice and stores every logit, tagged with the step, into every rank's region over
    NVLink; wait(out) reads (bounded) until all entries carry the step and copies the logits to out
    (fp32 [M][vocab]).

    exchange(handle) -> the handles of all ranks in rank order (e.g. torch_exchange).  For tests on
    one device, PeerGather.emulated builds `world` ranks in this process."""

    def __init__(self, ctx, rank: int, world: int, M: int, vocab: int, row_begin: int, exchange=None,
                 regions=None, own=None):
        from . import PeerGatherStruct
        self.ctx, self.rank, self.world, self.M, self.vocab = ctx, rank, world, M, vocab
        self.row_stride = vocab
        self.opened, self.owned = [], []
        if regions is None:
            nbytes = ctx.peer_region_bytes(M, self.row_stride)
            own, handle = ctx.peer_alloc(nbytes)
            self.owned.append(own)
            handles = exchange(handle) if world > 1 else [handle]
            regions = []
            for q, hq in enumerate(handles):
                if q == rank:
                    regions.append(own)
                else:
                    p = ctx.peer_open(hq)
                    self.opened.append(p)
                    regions.append(p)
        elif own is not None:
            self.owned.append(own)
        arr = (C.c_void_p * 8)(*(list(regions) + [None] * (8 - len(regions))))
        self.pg = PeerGatherStruct(world, rank, M, self.row_stride, row_begin, arr)

    @classmethod
    def emulated(cls, ctx, world: int, M: int, vocab: int) -> list["PeerGather"]:
        """`world` ranks in one process on ctx's device (their regions are plain device memory of
        this process, so no IPC)."""
        nbytes = ctx.peer_region_bytes(M, vocab)
        owns = [ctx.peer_alloc(nbytes)[0] for _ in range(world)]
        out = []
        for r in range(world):
            row0, _ = vocab_slice(r, world, vocab)
            out.append(cls(ctx, r, world, M, vocab, row0, regions=owns, own=owns[r]))
        return out

    def gather(self, w, x_dev, out_dev=None):
        """This rank's slice into every rank's buffer.  With out_dev the step completes inside the
        kernel (no wait call); without, wait() completes it."""
        self.ctx.gemm_peer_gather_async(w, x_dev, self.pg, out_dev)

    def wait(self, out_dev=None):
        self.ctx.peer_gather_wait_async(self.pg, out_dev)

    def close(self):
        for p in self.opened:
            self.ctx.peer_close(p)
        for p in self.owned:
            self.ctx.peer_free(p)
        self.opened, self.owned = [], []


def torch_exchange(handle: bytes, device) -> list[bytes]:
    """All ranks' IPC handles through torch.distributed (an all-gather of the 64 handle bytes)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(handle), dtype=torch.uint8, device=device)
    outs = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(outs, t)
    return [bytes(o.cpu().tolist()) for o in outs]
