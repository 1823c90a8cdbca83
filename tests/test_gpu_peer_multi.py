"""The in-GEMV all-gather across real GPUs (one process per GPU, IPC-mapped regions over NVLink):
every rank's gathered logits equal an unsharded GEMV bit for bit.  Skipped with fewer than 2
GPUs."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V, K, M, STEPS = 151936 // 8, 2560, 2, 4


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank: int, world: int, port: int, q, mode: str):
    import sys
    from datetime import timedelta
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist
    import npu880_mtk_npu_llm_runtime_b200 as kq
    from npu880_mtk_npu_llm_runtime_b200 import shard, synth
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        ctx = kq.Context(rank)
        w = synth.gen_weights(kq.TYPE_Q6_K, V, K, seed=90)
        r0, n = shard.vocab_slice(rank, world, V)
        Ws = ctx.upload(w[r0:r0 + n], kq.TYPE_Q6_K, n, K)
        Wf = ctx.upload(w, kq.TYPE_Q6_K, V, K)
        pg = shard.PeerGather(ctx, rank, world, M, V, r0, exchange=lambda h: shard.torch_exchange(h, dev))
        ok = True
        for step in range(STEPS):
            x = torch.from_numpy(synth.gen_activations(M, K, 91 + step).view(np.uint16).copy()).to(dev)
            ref = torch.zeros((M, V), dtype=torch.float32, device=dev)
            ctx.gemm_multi_async(x, M, K, ctx.make_tasks([dict(w=Wf, dst_f32=ref, dst_f32_stride=V)]))
            out = torch.full((M, pg.row_stride), float("nan"), dtype=torch.float32, device=dev)
            if mode == "in_kernel" or (mode == "mixed" and step % 2 == 0):
                pg.gather(Ws, x, out)  # completed by the GEMV's last CTAs
            else:
                pg.gather(Ws, x)
                pg.wait(out)
            ctx.synchronize()
            ok &= bool(np.array_equal(out[:, :V].cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32)))
        dist.barrier()
        pg.close()
        Ws.free()
        Wf.free()
        dist.destroy_process_group()
        q.put((rank, ok, ""))
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("mode", ["wait_kernel", "in_kernel", "mixed"])
@pytest.mark.parametrize("world", [2])
def test_peer_gather_two_processes(world, mode):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in sorted(results):
        assert ok, (rank, err)
