"""Benchmark of the B200 K-quant matmul path (one JSON line on rank 0).

Default workload: benchmark config 0 -- Q4_K x Q8_K GEMV, M=1, N=9728 rows, K=2560 (the FFN gate
shape of a 4B model), synthetic seeded GGUF blocks.  One step = one dispatch: the fp16
activation is quantized to Q8_K inside the kernel and the 9728 fp32 outputs are written.

  value  : weight GB/s over all ranks with inputs resident in HBM (kq_gemm_multi_async, steps
           captured in a CUDA graph, rotating weight copies holding more than 2.6x the 126 MB L2
           so every step streams its weights from HBM)
  e2e    : the same metric through the reference-facing C ABI with host buffers
           (kq_sdot_gemm_multi_dispatch: pinned fp16 input copied in, fp32 result written by
           the kernel into pinned host memory, one blocking call per step)
  roofline: algorithmic bytes per launch (weights + Q8_K activation + fp32 outputs) over the
           CUDA-event launch time, against the measured HBM copy bandwidth
  cpu_baseline: the reference's own dispatch on its thread pool (or the C restatement where the
           reference was not built), timed on this host's cores for a bounded sample
  clocks : SM clock and throttle reasons sampled by nvidia-smi during the timed region
  gpu_launches: kernels of this library launched inside the timed region

--config lm_head runs config 1 (Q6_K LM head, N=151936, K=2560) with vocab rows
sharded over the ranks and the logit slices all-gathered with NCCL, and (record p2p_gather) with
the gather inside the GEMV over NVLink.  --config ffn / prefill / decode run configs 2-4
(--tokens M; --ffn-fused 0 times the FFN block's four launches instead of the persistent kernel).
--impl reference times the reference engine's own CPU path (oracle/_ref, built from its
sources) on this host on the same workload.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                [--config gemv|lm_head|ffn|prefill|decode] [--tokens M]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC_GEMV = "Q4_K GEMV weight GB/s (% B200 HBM peak)"
METRIC_LM = "Q6_K LM-head GEMV weight GB/s (vocab-sharded, all-gathered)"
L2_BYTES = 126 * 1024 * 1024
DATA_DESC = "synthetic (seeded GGUF blocks per the benchmark configs' distributions; activations N(0,1) -> fp16)"
STEPS_DEFAULT = 300000


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(key, field="dram_bytes_per_launch"):
    """DRAM bytes of a kernel launch (or of one step) from the committed ncu summaries
    (profiles/traffic.json; each entry names the capture it comes from)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    v = d.get(key, {}).get(field)
    return None if v is None else float(v)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def __enter__(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.tmp, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.tmp is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.tmp.flush()
        rows = []
        with open(self.tmp.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def physical_gpu_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------- CPU baselines

def cpu_reference_gemv(n_rows, k, gtype, seconds=10.0, max_steps=None, warmup=1, single_thread=True):
    """The reference engine's own CPU path (sdot_gemm_multi_dispatch on its 4-thread pinned pool,
    turbo mode, scalar kernels on x86) over full GEMVs of the workload, and the same dispatch on one
    thread (its job function run by the calling thread alone).
    Returns a dict: value (weight GB/s of the pool), steps, seconds_per_step, kind, cores, sample,
    single_thread ({value, seconds_per_step, steps} or None)."""
    from npu880_mtk_npu_llm_runtime_b200 import synth
    from oracle.oracle import Reference, reference_available, Oracle
    w = synth.gen_weights(gtype, n_rows, k, seed=1234)
    x = synth.gen_activations(1, k, seed=1235)
    wbytes = w.nbytes

    def timed(fn, budget, cap):
        t0 = time.perf_counter()
        fn()
        t1 = time.perf_counter() - t0
        n = max(2, int(budget / max(t1, 1e-6)))
        if cap:
            n = min(n, cap)
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        return n, (time.perf_counter() - t0) / n

    if reference_available():
        R = Reference()
        R.init_pool()
        dst = np.zeros((1, n_rows), np.float16)
        R.turbo(True)
        for _ in range(warmup):
            R.dispatch(x, [(gtype, w, dst, None)])
        steps, sec = timed(lambda: R.dispatch(x, [(gtype, w, dst, None)]), seconds, max_steps)
        R.turbo(False)
        one = None
        if single_thread:
            n1, s1 = timed(lambda: R.dispatch_1thread(x, [(gtype, w, dst, None)]), seconds / 3, max_steps)
            one = {"value": round(wbytes / s1 / 1e9, 4), "unit": "GB/s", "cores": 1, "steps": n1,
                   "seconds_per_step": s1,
                   "sample": f"{n1} full GEMVs through the same dispatch with its job function "
                             f"(exec_sdot_job_work_stealing) run on one thread"}
        return {"value": wbytes / sec / 1e9, "steps": steps, "seconds_per_step": sec, "kind": "reference",
                "cores": R.pool_threads,
                "sample": f"{steps} full GEMVs (N={n_rows}, K={k}) through the reference's sdot_gemm_multi_dispatch "
                          f"on its {R.pool_threads}-thread pool (scalar x86 kernels, turbo mode)",
                "single_thread": one}
    O = Oracle()
    act = O.quantize_q8k(x)
    steps, sec = timed(lambda: O.gemm(gtype, w, k, act), seconds, max_steps)
    return {"value": wbytes / sec / 1e9, "steps": steps, "seconds_per_step": sec, "kind": "port", "cores": 1,
            "sample": f"{steps} full GEMVs (N={n_rows}, K={k}) through the oracle's scalar C restatement, 1 thread",
            "single_thread": None}


# ---------------------------------------------------------------------------- timing helpers

GRAPH_MAX = 1000  # launches per captured graph


def graph_timed(stream, step, steps, warmup, world, per_step_launches=1):
    """Time `steps` calls of step(i) on the device, hot: one eager call configures the kernels,
    then a CUDA graph holds the `warmup` untimed steps, a timing event, the `steps` timed steps and
    a second event, so the timed steps start right after warm-up steps with the GPU busy (no idle
    gap, no graph boundary inside the timed region).  The first event is recorded on a side branch
    of the graph (it fires when the warm-up steps have completed) so that the first timed launch
    keeps its programmatic-dependent-launch edge to the last warm-up launch, as every later one
    does.  Beyond GRAPH_MAX steps the timed steps are replayed from graphs of at most GRAPH_MAX
    steps.  Returns seconds (max over ranks)."""
    import torch
    import torch.distributed as dist
    with torch.cuda.stream(stream):
        step(0)
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True, external=True)
    ev1 = torch.cuda.Event(enable_timing=True, external=True)
    graphs = []
    try:
        if steps <= GRAPH_MAX:
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(device=stream.device)
            fork, join = torch.cuda.Event(), torch.cuda.Event()
            with torch.cuda.graph(g, stream=stream):
                for i in range(warmup):
                    step(i)
                fork.record(stream)
                side.wait_event(fork)
                ev0.record(side)
                for i in range(steps):
                    step(warmup + i)
                ev1.record(stream)
                join.record(side)
                stream.wait_event(join)
            graphs.append(g)
            plan = [g]
        else:
            gw = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gw, stream=stream):
                for i in range(warmup):
                    step(i)
                ev0.record()
            graphs.append(gw)
            full, rem = divmod(steps, GRAPH_MAX)
            gt = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gt, stream=stream):
                for i in range(GRAPH_MAX):
                    step(warmup + i)
            graphs.append(gt)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for i in range(rem):
                    step(warmup + i)
                ev1.record()
            graphs.append(gr)
            plan = [gw] + [gt] * full + [gr]
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for g in plan:
                g.replay()
        ev1.synchronize()
        dt = ev0.elapsed_time(ev1) / 1e3
    finally:
        torch.cuda.synchronize()
        del graphs[:]
    t = torch.tensor([dt], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def e2e_timed(stream, call, steps, warmup, world):
    """Blocking host-buffer calls: `warmup` untimed calls right before `steps` timed ones, CUDA
    events on the context stream around the timed calls.  Returns seconds (max over ranks)."""
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    for i in range(warmup):
        call(i)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        call(warmup + i)
    e1.record(stream)
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------- our arm: configs 0 and 1

def gemv_config(world, n_copies=None, wbytes=None):
    """The `config` record both arms print for config 0 (the reference arm without run facts)."""
    return {"workload": "config0: Q4_K x Q8_K GEMV M=1 N=9728 K=2560", "m": 1, "n": 9728, "k": 2560,
            "weight_bytes_per_step_per_rank": 14008320,
            "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2: rotating weight copies of > 2x126 MB L2 per rank",
            "timing": "CUDA graph: warm-up steps, event, timed steps, event (one replay); CUDA events"}


def lm_config(world):
    return {"workload": "config1: Q6_K LM head M=1 N=151936 K=2560, vocab rows sharded, "
                        "NCCL all-gather of fp32 logit slices",
            "m": 1, "n": 151936, "k": 2560, "weight_bytes_per_step_per_rank": None,
            "parallelism": f"vocab-shard x{world}",
            "l2": "inputs larger than L2: rotating weight copies of > 2x126 MB L2 per rank",
            "timing": "CUDA graph of (GEMV + NCCL all-gather) steps: warm-up steps, event, timed steps, event; "
                      "max over ranks"}


def lm_head_sharded(ctx, args, rank, world, dev, stream, steps, warmup, want_argmax=True):
    """Config 1 on `world` ranks: each rank streams its contiguous slice of the 151,936 Q6_K vocab
    rows (GEMV, fp32 logits written straight into its chunk of the gather buffer), then one NCCL
    all-gather of the logit slices (in place); GEMV + all-gather captured in CUDA graphs.  With
    want_argmax also the argmax-only exchange: each rank's fused GEMV argmax, an all-gather of one
    (value, row) pair per rank, merged on the device (largest value, first row on ties)."""
    import torch
    import torch.distributed as dist
    import npu880_mtk_npu_llm_runtime_b200 as kq
    from npu880_mtk_npu_llm_runtime_b200 import shard, synth
    V, K = 151936, 2560
    row0, rows = shard.vocab_slice(rank, world, V)
    chunk = (V + world - 1) // world
    w_host = synth.gen_weights(kq.TYPE_Q6_K, V, K, seed=4321)[row0:row0 + rows]
    x_host = synth.gen_activations(1, K, seed=4322)
    wbytes = w_host.nbytes
    raw = torch.from_numpy(np.ascontiguousarray(w_host)).to(dev)
    n_copies = max(2, math.ceil(2.6 * L2_BYTES / max(1, wbytes)))
    Ws = [ctx.upload_device(raw, kq.TYPE_Q6_K, rows, K) for _ in range(n_copies)]
    del raw
    x = torch.from_numpy(x_host.view(np.uint16).copy()).to(dev)
    gather = torch.zeros((world * chunk,), dtype=torch.float32, device=dev)
    mine = gather[rank * chunk:(rank + 1) * chunk]
    tasks = [ctx.make_tasks([dict(w=Ws[i], dst_f32=mine[:rows].view(1, rows), dst_f32_stride=rows)])
             for i in range(n_copies)]

    def step(i):
        ctx.gemm_multi_async(x, 1, K, tasks[i % n_copies])
        if world > 1:
            dist.all_gather_into_tensor(gather, mine)

    dt = graph_timed(stream, step, steps, warmup, world)
    total = torch.tensor([float(wbytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.SUM)
    value = float(total.item()) * steps / dt / 1e9
    rec = {"value": round(value, 1), "unit": "GB/s", "ms_per_step": round(dt / steps * 1e3, 6), "steps": steps,
           "warmup": warmup, "n_gpus": world, "rows_per_rank": chunk, "weight_bytes_per_rank": wbytes,
           "gather_bytes_per_rank": chunk * 4}
    # the all-gather inside the GEMV: its epilogue stores every logit into every rank's gather
    # buffer over NVLink, then a bounded wait for all ranks' slices copies the gathered logits out
    pg = shard.PeerGather(ctx, rank, world, 1, V, row0,
                          exchange=(lambda h: shard.torch_exchange(h, dev)) if world > 1 else None)
    p2p_out = torch.zeros((1, pg.row_stride), dtype=torch.float32, device=dev)

    def step_p(i):  # the step completes inside the GEMV (its last CTAs collect the other ranks' rows)
        pg.gather(Ws[i % n_copies], x, p2p_out)

    def step_w(i):  # the same with a separate wait kernel
        pg.gather(Ws[i % n_copies], x)
        pg.wait(p2p_out)

    dtw = graph_timed(stream, step_w, steps, warmup, world)
    dtp = graph_timed(stream, step_p, steps, warmup, world)
    torch.cuda.synchronize()
    same = bool(torch.equal(p2p_out[0, :V], gather[:V]))
    rec["p2p_gather"] = {"value": round(float(total.item()) * steps / dtp / 1e9, 1), "unit": "GB/s",
                         "ms_per_step": round(dtp / steps * 1e3, 6), "equal_to_nccl_gather": same,
                         "how": "GEMV epilogue stores each logit into every rank's buffer over NVLink as one 64-bit "
                                "(step, fp32) entry; the GEMV's last CTAs read the other ranks' entries until all carry "
                                "the step and write the fp32 logits out",
                         "with_wait_kernel": {"ms_per_step": round(dtw / steps * 1e3, 6),
                                              "value": round(float(total.item()) * steps / dtw / 1e9, 1)}}
    if world > 1:
        dist.barrier()
    pg.close()
    if want_argmax:
        toks = torch.zeros((1,), dtype=torch.int32, device=dev)
        vals = torch.zeros((1,), dtype=torch.float32, device=dev)
        pair = torch.zeros((2,), dtype=torch.float32, device=dev)
        pairs = torch.zeros((world, 2), dtype=torch.float32, device=dev)
        best = torch.zeros((2,), dtype=torch.float32, device=dev)

        def step_a(i):
            ctx.lm_head_argmax_async(Ws[i % n_copies], x, 1, None, None, toks, vals)
            pair[0:1].copy_(vals)
            pair[1:2].copy_((toks + row0).float())   # global row (< 2^24: exact in fp32)
            if world > 1:
                dist.all_gather_into_tensor(pairs.view(-1), pair)
            else:
                pairs[0].copy_(pair)
            r = torch.argmax(pairs[:, 0]).view(1)        # first rank with the maximum = first row
            best.copy_(torch.index_select(pairs, 0, r).view(2))

        dta = graph_timed(stream, step_a, steps, warmup, world)
        rec["argmax_exchange"] = {"value": round(float(total.item()) * steps / dta / 1e9, 1), "unit": "GB/s",
                                  "ms_per_step": round(dta / steps * 1e3, 6), "exchange_bytes_per_rank": 8}
    for W in Ws:
        W.free()
    return rec


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import npu880_mtk_npu_llm_runtime_b200 as kq
    from npu880_mtk_npu_llm_runtime_b200 import build as kqbuild, synth

    kqbuild.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    ctx = kq.Context(local_rank)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    warmup = max(3, args.warmup)
    steps = args.steps
    peak, peak_kind = measured_peaks()
    clk = ClockSampler(physical_gpu_index(local_rank))
    clk.__enter__()  # sampling runs from before the warm-up to after the timed steps

    if args.config == "lm_head":
        rec = lm_head_sharded(ctx, args, rank, world, dev, stream, steps, warmup)
        clk.__exit__()
        clocks = clk.summary()
        result = None
        if rank == 0:
            cfg = lm_config(world)
            cfg["weight_bytes_per_step_per_rank"] = rec["weight_bytes_per_rank"]
            avg_s = rec["ms_per_step"] / 1e3
            algo = rec["weight_bytes_per_rank"] + rec["rows_per_rank"] * 4 + 2920
            result = {
                "metric": METRIC_LM, "value": rec["value"], "unit": "GB/s", "n_gpus": world, "steps": steps,
                "warmup": warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int8", "data": DATA_DESC, "config": cfg,
                "roofline": {"bound": "hbm", "achieved": round(algo / avg_s / 1e9, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(algo / avg_s / 1e9 / peak, 4), "peak_source": peak_kind,
                             "traffic": ncu_traffic("gemv_q6k_lmhead"),
                             "note": "step time includes the all-gather at N > 1"},
                "argmax_exchange": rec.get("argmax_exchange"), "p2p_gather": rec.get("p2p_gather"),
                "cpu_baseline": None, "clocks": clocks,
                "e2e": None, "gpu_launches": steps * (1 + (world > 1)),
            }
        ctx.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return result

    # ---------------- config 0: Q4_K GEMV, replicated on every rank
    gtype, N, K = kq.TYPE_Q4_K, 9728, 2560
    w_host = synth.gen_weights(gtype, N, K, seed=1234)
    x_host = synth.gen_activations(1, K, seed=1235)
    wbytes = w_host.nbytes
    raw = torch.from_numpy(np.ascontiguousarray(w_host)).to(dev)
    n_copies = max(2, math.ceil(2.6 * L2_BYTES / max(1, wbytes)))
    Ws = [ctx.upload_device(raw, gtype, N, K) for _ in range(n_copies)]
    del raw
    x = torch.from_numpy(x_host.view(np.uint16).copy()).to(dev)
    out = torch.zeros((n_copies, N), dtype=torch.float32, device=dev)
    tasks = [ctx.make_tasks([dict(w=Ws[i], dst_f32=out[i:i + 1], dst_f32_stride=N)]) for i in range(n_copies)]

    def step(i):
        ctx.gemm_multi_async(x, 1, K, tasks[i % n_copies])

    dt = graph_timed(stream, step, steps, warmup, world)
    dt_local = dt  # max over ranks already; the roofline uses the same launch time
    total_wbytes = torch.tensor([float(wbytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total_wbytes, op=dist.ReduceOp.SUM)
    value = float(total_wbytes.item()) * steps / dt / 1e9
    ms_per_step = dt / steps * 1e3

    # roofline of the GEMV kernel: algorithmic bytes per launch / launch duration
    act_bytes = (K // 256) * 292            # Q8_K activation: 292 B per 256 values (2,920 B at K=2560)
    algo = wbytes + act_bytes + N * 4
    achieved = algo / (dt_local / steps) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": peak_kind, "traffic": ncu_traffic("gemv_q4k_cfg0"),
            "algorithmic_bytes_per_launch": algo}

    # e2e through the reference-facing C ABI with host buffers (blocking calls)
    e2e_steps = min(steps, args.e2e_steps)
    xp = torch.from_numpy(x_host.view(np.uint16).copy()).pin_memory()
    op = torch.zeros((1, N), dtype=torch.float32).pin_memory()
    xp_np = xp.numpy().view(np.float16)
    op_np = op.numpy()
    htasks = [ctx.make_host_tasks([dict(w=Ws[i], dst_f32=op_np)]) for i in range(n_copies)]
    te = e2e_timed(stream, lambda i: ctx.sdot_gemm_multi_dispatch(xp_np, htasks[i % n_copies]), e2e_steps,
                   max(warmup, 100), world)
    e2e_value = float(total_wbytes.item()) * e2e_steps / te / 1e9
    for W in Ws:
        W.free()

    # the sharded LM head (config 1) at this rank count, as a nested record
    lm = None
    if not args.no_lm_head:
        lm = lm_head_sharded(ctx, args, rank, world, dev, stream, min(steps, 2000), warmup)
    clk.__exit__()
    clocks = clk.summary()

    result = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            c = cpu_reference_gemv(N, K, gtype, seconds=args.cpu_seconds)
            cpu = {"value": round(c["value"], 4), "unit": "GB/s", "cores": c["cores"], "kind": c["kind"],
                   "sample": c["sample"], "seconds_per_step": c["seconds_per_step"],
                   "single_thread": c["single_thread"]}
        cfg = gemv_config(world)
        cfg["weight_bytes_per_step_per_rank"] = wbytes
        cfg["l2"] = f"inputs larger than L2: {n_copies} rotating weight copies ({n_copies * wbytes / 2**20:.0f} MiB > 2x126 MB L2)"
        if lm is not None:
            cfg["lm_head_sharded"] = dict(lm, workload=lm_config(world)["workload"],
                                          parallelism=f"vocab-shard x{world}")
        result = {
            "metric": METRIC_GEMV, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": DATA_DESC, "config": cfg,
            "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": int(x_host.nbytes), "d2h_bytes_per_step": int(N * 4),
                    "api": "kq_sdot_gemm_multi_dispatch (host buffers, blocking)",
                    "scope": "one blocking call per step; max over ranks"},
            "gpu_launches": steps,
        }
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ---------------------------------------------------------------------------- stack configs

METRIC_FFN = "tree-verify FFN block weight GB/s (Q4_K gate/up, Q6_K down)"
METRIC_PREFILL = "prefill GEMM TOPS (36-layer Q4_K_M stack, int8 tensor cores)"
METRIC_DECODE = "batched decode tok/s (64 sequences, 36-layer Q5_K/Q8_0 stack + sharded LM head)"

HIDDEN, FFN_DIM, Q_DIM, KV_DIM, VOCAB = 2560, 9728, 4096, 1024, 151936


def stack_layout(kind):
    """(name, type, rows, K) of one layer: config 3 (Q4_K_M prefill stack) or config 4 (Q5_K/Q8_0 decode stack)."""
    from npu880_mtk_npu_llm_runtime_b200 import synth as sy
    if kind == "prefill":
        a, b = sy.TYPE_Q4_K, sy.TYPE_Q6_K
        return [("q", a, Q_DIM, HIDDEN), ("k", a, KV_DIM, HIDDEN), ("v", b, KV_DIM, HIDDEN), ("o", a, HIDDEN, Q_DIM),
                ("gate", a, FFN_DIM, HIDDEN), ("up", a, FFN_DIM, HIDDEN), ("down", b, HIDDEN, FFN_DIM)]
    a, b = sy.TYPE_Q5_K, sy.TYPE_Q8_0
    return [("q", a, Q_DIM, HIDDEN), ("k", b, KV_DIM, HIDDEN), ("v", b, KV_DIM, HIDDEN), ("o", a, HIDDEN, Q_DIM),
            ("gate", a, FFN_DIM, HIDDEN), ("up", a, FFN_DIM, HIDDEN), ("down", b, HIDDEN, FFN_DIM)]


def time_device(stream, step, steps, warmup, gpu_index, graph=True, world=1):
    """Time `steps` calls of step(i) after `warmup` untimed ones, with the clock sampler running
    from before the warm-up.  graph: graph_timed (warm-up and timed steps in one CUDA graph).
    Eager: the ranks meet at a barrier, then the warm-up steps, a timing event and the timed steps
    are enqueued back to back, so the timed steps start with the GPU busy.  Returns (seconds, max
    over ranks; clock summary)."""
    import torch
    import torch.distributed as dist
    clk = ClockSampler(gpu_index)
    clk.__enter__()
    try:
        if graph:
            dt = graph_timed(stream, step, steps, warmup, world)
        else:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                for i in range(warmup):
                    step(i)
                e0.record(stream)
                for i in range(steps):
                    step(warmup + i)
                e1.record(stream)
            e1.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device="cuda")
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
    finally:
        clk.__exit__()
    return dt, clk.summary()


def run_stack(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import npu880_mtk_npu_llm_runtime_b200 as kq
    from npu880_mtk_npu_llm_runtime_b200 import build as kqbuild, shard, synth

    kqbuild.build()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    ctx = kq.Context(local_rank)
    stream = torch.cuda.Stream(device=dev)
    ctx.set_stream(stream.cuda_stream)
    gpu = physical_gpu_index(local_rank)
    peak_hbm, peak_kind = measured_peaks()
    result = None

    def qact(x16_dev, M, K, gtype):
        if gtype == synth.TYPE_Q8_0:
            q = torch.zeros(kq.q8_0_bytes(M, K), dtype=torch.uint8, device=dev)
            ctx.quantize_q8_0_async(x16_dev, M, K, q)
            return None, q
        q = torch.zeros(kq.q8k_bytes(M, K), dtype=torch.uint8, device=dev)
        ctx.quantize_q8k_async(x16_dev, M, K, q)
        return q, None

    if args.config == "ffn":
        # config 2: RMSNorm -> {gate, up} Q4_K -> SwiGLU -> down Q6_K + residual, M draft tokens
        # (M in the hundreds or thousands: the batched prefill FFN).  One GPU: the library's FFN
        # entry point.  N GPUs: rows sharded (shard.RowShardedFfn, two NCCL all-gathers per step)
        M = args.tokens or 8
        per_set = [synth.gen_weights(synth.TYPE_Q4_K, FFN_DIM, HIDDEN, 2001), synth.gen_weights(synth.TYPE_Q4_K, FFN_DIM, HIDDEN, 2002),
                   synth.gen_weights(synth.TYPE_Q6_K, HIDDEN, FFN_DIM, 2003)]
        wbytes = sum(w.nbytes for w in per_set)
        plan = shard.FfnShardPlan(HIDDEN, FFN_DIM, world)
        c0, C = plan.inter(rank)
        r0, R = plan.hid(rank)
        local = [per_set[0][c0:c0 + C], per_set[1][c0:c0 + C], per_set[2][r0:r0 + R]]
        rank_wbytes = sum(w.nbytes for w in local)
        n_sets = max(2, math.ceil(2.2 * L2_BYTES / rank_wbytes))
        shapes = [(synth.TYPE_Q4_K, C, HIDDEN), (synth.TYPE_Q4_K, C, HIDDEN), (synth.TYPE_Q6_K, R, FFN_DIM)]
        sets = [tuple(ctx.upload(w, t, r, k) for w, (t, r, k) in zip(local, shapes)) for _ in range(n_sets)]
        x16 = synth.gen_activations(M, HIDDEN, 2004)
        gamma = (synth.gen_gamma(HIDDEN, 2005) * np.float16(0.1)).astype(np.float16)
        x = torch.from_numpy(x16.view(np.uint16).copy()).to(dev).view(torch.float16).view(M, HIDDEN)
        gm = torch.from_numpy(gamma.view(np.uint16).copy()).to(dev)
        out = torch.zeros((M, HIDDEN), dtype=torch.float16, device=dev)
        ctx.set_option("ffn_fused", args.ffn_fused)
        fused = bool(args.ffn_fused) and M <= 2  # the persistent kernel covers 1-2 tokens of these types
        if world == 1:
            def step(i):
                g_, u_, d_ = sets[i % n_sets]
                ctx.run_ffn_async(g_, u_, d_, M, x, gm, out)
            launches = 1 if fused else 4
        else:
            rk = shard.RowShardedFfn(ctx, plan, rank, M, dev)
            tks = [rk.tasks(*st_, x) for st_ in sets]

            def gather(o, i_):
                dist.all_gather_into_tensor(o, i_)

            def step(i):
                gu, dn = tks[i % n_sets]
                rk.forward(x, gm, out, gu, dn, gather)
            launches = 6

        steps = args.steps
        warmup = max(3, args.warmup)
        dt, clocks = time_device(stream, step, steps, warmup, gpu, world=world)
        value = wbytes * steps / dt / 1e9
        ops = 2.0 * M * (2 * FFN_DIM * HIDDEN + HIDDEN * FFN_DIM)
        # e2e with host buffers: one GPU, the blocking C-ABI call kq_run_ffn; N GPUs, each rank
        # copies the pinned input in, runs its sharded step and copies the assembled output out
        e2e_steps = min(steps, 200)
        if world == 1:
            xp = np.ascontiguousarray(x16)
            e2e_dt = e2e_timed(stream, lambda i: ctx.run_ffn(*sets[i % n_sets], xp, gamma), e2e_steps, 20, world)
            e2e_api = "kq_run_ffn (host buffers, blocking)"
        else:
            xh = torch.from_numpy(x16.view(np.uint16).copy()).pin_memory()
            oh = torch.zeros((M, HIDDEN), dtype=torch.float16).pin_memory()

            def call(i):
                with torch.cuda.stream(stream):
                    x.view(torch.uint16).copy_(xh.view(M, HIDDEN), non_blocking=True)
                    step(i)
                    oh.copy_(out, non_blocking=True)
                stream.synchronize()
            e2e_dt = e2e_timed(stream, call, e2e_steps, 20, world)
            e2e_api = "pinned input copied in, row-sharded step (library calls + NCCL), output copied out"
        cpu = None
        if not args.no_cpu_baseline and rank == 0 and world == 1 and M <= 64:
            from oracle.oracle import Oracle
            O = Oracle()
            t0 = time.perf_counter()
            O.ffn(per_set[0], synth.TYPE_Q4_K, per_set[1], synth.TYPE_Q4_K, per_set[2], synth.TYPE_Q6_K, HIDDEN, FFN_DIM, x16, gamma)
            sec = time.perf_counter() - t0
            cpu = {"value": round(wbytes / sec / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                   "sample": f"1 FFN block at M={M} through the oracle's C restatement of the reference's SDOT "
                             f"FFN sequence (ENG:8283-8298; its dispatch limit K <= 9216 excludes down, K = 9728)",
                   "seconds_per_step": sec}
        per_rank = rank_wbytes * steps / dt / 1e9
        result = {
            "metric": METRIC_FFN, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(dt / steps * 1e3, 6), "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong", "vs_baseline": None, "dtype": "int8",
            "data": DATA_DESC,
            "config": {"workload": f"config2: FFN block M={M}, hidden 2560, intermediate 9728"
                                   + (" (batched prefill FFN)" if M > 64 else " (tree verify)"),
                       "m": M, "weight_bytes_per_step": wbytes, "weight_bytes_per_step_per_rank": rank_wbytes,
                       "form": ("one persistent kernel (kq_ffn_fused)" if fused and world == 1 else
                                "RMSNorm+Q8_K, gate/up, SwiGLU+Q8_K, down+residual launches"),
                       "tops": round(ops * steps / dt / 1e12, 3),
                       "l2": f"{n_sets} rotating weight sets per rank ({n_sets * rank_wbytes / 2**20:.0f} MiB > 2x126 MB L2)",
                       "parallelism": "replicas x1" if world == 1 else f"row-shard x{world}",
                       "timing": "CUDA graph: warm-up steps, event, timed steps, event"
                                 + ("" if world == 1 else " (NCCL all-gathers captured); max over ranks")},
            "roofline": ({"bound": "hbm", "achieved": round(per_rank, 1), "peak": peak_hbm, "unit": "GB/s",
                          "frac": round(per_rank / peak_hbm, 4), "peak_source": peak_kind,
                          "traffic": ncu_traffic(f"ffn_m{M}", "dram_bytes_per_step") if world == 1 else None,
                          "note": "weight bytes of this rank's share per step time (the whole block at 1 GPU); "
                                  "traffic = DRAM bytes of one whole step (all its kernels) from the ncu summary"}
                         if M <= 64 else ffn_tensor_roofline(ops * steps / dt / 1e12 / world, local_rank)),
            "cpu_baseline": cpu, "clocks": clocks,
            "e2e": {"value": round(wbytes * e2e_steps / e2e_dt / 1e9, 2), "unit": "GB/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": int(x16.nbytes + (gamma.nbytes if world == 1 else 0)),
                    "d2h_bytes_per_step": int(x16.nbytes), "api": e2e_api},
            "gpu_launches": steps * launches,
        }
        for st_ in sets:
            for w_ in st_:
                w_.free()

    elif args.config in ("prefill", "decode"):
        # configs 3 and 4: the decoder stack's matrix products chained layer by layer through the
        # producers.  Per layer: RMSNorm + Q8_K (and Q8_0 for Q8_0 weights) -> q / k / v (one
        # dispatch) -> o over q's output with the residual (the attention core is outside the
        # path, so q's output stands in for its result) -> the FFN block (RMSNorm, gate / up,
        # SwiGLU, down + residual).  Config 3 (prefill, M tokens): at N GPUs the FFN rows are
        # sharded (shard.RowShardedFfn), the projections replicated.  Config 4 (decode, 64
        # sequences): the sequences split over the ranks, then the final RMSNorm, an all-gather of
        # the normalised rows, each rank's vocabulary slice of the LM head for all rows, and the
        # per-row (value, row) pairs all-gathered and merged on the device.
        prefill = args.config == "prefill"
        kind = "prefill" if prefill else "decode"
        L = args.layers
        SEQ = 64
        M = (args.tokens or 2048) if prefill else SEQ // world
        sharded_ffn = prefill and world > 1
        layout = stack_layout(kind)
        host = {n: synth.gen_weights(t, r, k, (3000 if prefill else 4000) + i) for i, (n, t, r, k) in enumerate(layout)}
        types = {n: t for (n, t, r, k) in layout}
        plan = shard.FfnShardPlan(HIDDEN, FFN_DIM, world)
        c0, C = plan.inter(rank)
        r0, R = plan.hid(rank)
        rank_wbytes = 0
        layers = []
        for _ in range(L):
            lay = {}
            for (n, t, r, k) in layout:
                w_ = host[n]
                if sharded_ffn and n in ("gate", "up"):
                    w_, r = w_[c0:c0 + C], C
                elif sharded_ffn and n == "down":
                    w_, r = w_[r0:r0 + R], R
                lay[n] = ctx.upload(w_, t, r, k)
                rank_wbytes += w_.nbytes
            layers.append(lay)
        g_attn = torch.from_numpy((synth.gen_gamma(HIDDEN, 3900) * np.float16(0.1)).astype(np.float16).view(np.uint16).copy()).to(dev)
        g_ffn = torch.from_numpy((synth.gen_gamma(HIDDEN, 3901) * np.float16(0.1)).astype(np.float16).view(np.uint16).copy()).to(dev)
        f16 = torch.float16
        h_a = torch.zeros((M, HIDDEN), dtype=f16, device=dev)
        h_b = torch.zeros_like(h_a)
        h_mid = torch.zeros_like(h_a)
        xn = torch.zeros_like(h_a)
        qx = torch.zeros(kq.q8k_bytes(M, HIDDEN), dtype=torch.uint8, device=dev)
        need_q80 = any(types[n] == synth.TYPE_Q8_0 for n in ("q", "k", "v"))
        qx0 = torch.zeros(kq.q8_0_bytes(M, HIDDEN), dtype=torch.uint8, device=dev) if need_q80 else None
        qo = torch.zeros((M, Q_DIM), dtype=f16, device=dev)
        ko = torch.zeros((M, KV_DIM), dtype=f16, device=dev)
        vo = torch.zeros((M, KV_DIM), dtype=f16, device=dev)
        x_host = synth.gen_activations(M, HIDDEN, (3100 if prefill else 4300) + rank)
        x_dev = torch.from_numpy(x_host.view(np.uint16).copy()).to(dev).view(f16).view(M, HIDDEN)
        qkv = [ctx.make_tasks([dict(w=lay["q"], dst=qo), dict(w=lay["k"], dst=ko), dict(w=lay["v"], dst=vo)])
               for lay in layers]
        o_tasks = [[ctx.make_tasks([dict(w=lay["o"], dst=dst, residual=src)]) for (src, dst) in ((h_a, h_mid), (h_b, h_mid))]
                   for lay in layers]
        rk = None
        if sharded_ffn:
            rk = shard.RowShardedFfn(ctx, plan, rank, M, dev)
            ffn_tasks = [[rk.tasks(lay["gate"], lay["up"], lay["down"], h_mid)] for lay in layers]

            def gather(o, i_):
                dist.all_gather_into_tensor(o, i_)

        def run_layers():
            src, dst = h_a, h_b
            for li, lay in enumerate(layers):
                ctx.rmsnorm_q8k_async(src, g_attn, xn, M, HIDDEN, qx)
                if need_q80:
                    ctx.quantize_q8_0_async(xn, M, HIDDEN, qx0)
                ctx.gemm_multi_q8_async(qx, qx0, M, HIDDEN, qkv[li])
                ctx.gemm_multi_async(qo, M, Q_DIM, o_tasks[li][0 if src is h_a else 1])
                if rk is not None:
                    gu, dn = ffn_tasks[li][0]
                    rk.forward(h_mid, g_ffn, dst, gu, dn, gather)
                else:
                    ctx.run_ffn_async(lay["gate"], lay["up"], lay["down"], M, h_mid, g_ffn, dst)
                src, dst = dst, src
            return src

        if prefill:
            def step(i):
                h_a.copy_(x_dev)
                run_layers()
            launches_per_step = L * (5 + (7 if sharded_ffn else 4)) + 1
        else:
            v0, vrows = shard.vocab_slice(rank, world, VOCAB)
            lm_host = synth.gen_weights(synth.TYPE_Q6_K, VOCAB, HIDDEN, 4100)[v0:v0 + vrows]
            lm = ctx.upload(lm_host, synth.TYPE_Q6_K, vrows, HIDDEN)
            rank_wbytes += lm_host.nbytes
            g_out = torch.from_numpy((synth.gen_gamma(HIDDEN, 3902) * np.float16(0.1)).astype(np.float16).view(np.uint16).copy()).to(dev)
            nrm = torch.zeros((M, HIDDEN), dtype=f16, device=dev)
            nrm_all = torch.zeros((SEQ, HIDDEN), dtype=f16, device=dev)
            toks = torch.zeros((SEQ,), dtype=torch.int32, device=dev)
            vals = torch.zeros((SEQ,), dtype=torch.float32, device=dev)
            pair = torch.zeros((2, SEQ), dtype=torch.float32, device=dev)
            pair_all = torch.zeros((world * 2, SEQ), dtype=torch.float32, device=dev)
            best = torch.zeros((SEQ,), dtype=torch.int64, device=dev)
            cols = torch.arange(SEQ, device=dev)

            def step(i):
                h_a.copy_(x_dev)
                last = run_layers()
                ctx.rmsnorm_q8k_async(last, g_out, nrm, M, HIDDEN, qx)   # final norm of this rank's rows
                if world > 1:
                    dist.all_gather_into_tensor(nrm_all, nrm)
                else:
                    nrm_all.copy_(nrm)
                ctx.lm_head_argmax_async(lm, nrm_all, SEQ, None, None, toks, vals)
                pair[0].copy_(vals)
                pair[1].copy_((toks + v0).float())          # global rows (< 2^24: exact in fp32)
                if world > 1:
                    dist.all_gather_into_tensor(pair_all, pair)
                else:
                    pair_all.copy_(pair)
                pv = pair_all.view(world, 2, SEQ)
                r_ = torch.argmax(pv[:, 0, :], dim=0)       # first rank with the maximum = first row
                best.copy_(pv[:, 1, :][r_, cols].long())
            launches_per_step = L * (5 + 4 + (1 if need_q80 else 0)) + 4

        steps = args.steps
        warmup = max(3, args.warmup)
        dt, clocks = time_device(stream, step, steps, warmup, gpu, graph=not prefill, world=world)
        # e2e with host buffers: the step's input rows copied in from pinned memory, the result
        # (prefill: the last hidden rows; decode: the 64 next tokens) copied out
        xh = torch.from_numpy(x_host.view(np.uint16).copy()).pin_memory()
        if prefill:
            oh = torch.zeros((M, HIDDEN), dtype=torch.float16).pin_memory()
            d2h = M * HIDDEN * 2
        else:
            oh = torch.zeros((SEQ,), dtype=torch.int64).pin_memory()
            d2h = SEQ * 8

        def call(i):
            with torch.cuda.stream(stream):
                x_dev.view(torch.uint16).copy_(xh.view(M, HIDDEN), non_blocking=True)
                step(i)
                oh.copy_(h_a if (prefill and L % 2 == 0) else (h_b if prefill else best), non_blocking=True)
            stream.synchronize()
        e2e_steps = max(1, min(steps, 3 if prefill else 20))
        e2e_dt = e2e_timed(stream, call, e2e_steps, 1, world)
        ops = 2.0 * (M * world if not prefill else M) * sum(r * k for (_, _, r, k) in layout) * L
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            from oracle.oracle import Reference, reference_available, Oracle
            rows_s, Ms = (256, 32) if prefill else (128, 8)
            t_layer = 0.0
            kind_s = "port"
            for (n, t, r, k) in layout:
                a_ = Oracle().act_for(t, synth.gen_activations(Ms, k, 3200))
                t0 = time.perf_counter()
                if reference_available() and k <= 9216:
                    Reference().gemm(t, host[n][:rows_s], k, a_)
                    kind_s = "reference"
                else:
                    Oracle().gemm(t, host[n][:rows_s], k, a_)
                t_layer += (time.perf_counter() - t0) * r / rows_s
            if prefill:
                cpu = {"value": round(2.0 * Ms * sum(r * k for (_, _, r, k) in layout) / t_layer / 1e12, 6),
                       "unit": "TOPS", "cores": 1, "kind": kind_s,
                       "sample": f"first {rows_s} rows of every matrix of one layer at {Ms} tokens through the "
                                 f"reference's row kernels (sdot_row_<type>_batch, scalar x86; the down projection, "
                                 f"K = 9728 > the reference's 9216, through the oracle), 1 thread, scaled to full rows"}
            else:
                cpu = {"value": round(Ms / (t_layer * L), 4), "unit": "tok/s", "cores": 1, "kind": kind_s,
                       "sample": f"first {rows_s} rows of every matrix of one layer at {Ms} tokens through the "
                                 f"reference's row kernels (the 9728-value down projection through the oracle), "
                                 f"1 thread, scaled to full rows and {L} layers; LM head not included"}
        if rank == 0:
            common = {"n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": round(dt / steps * 1e3, 4),
                      "higher_is_better": True, "vs_baseline": None, "dtype": "int8", "data": DATA_DESC,
                      "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": steps * launches_per_step}
            if prefill:
                value = ops * steps / dt / 1e12
                peak_int8, peak_int8_src = measured_int8_tops(local_rank)
                result = dict(common, **{
                    "metric": METRIC_PREFILL, "value": round(value, 2), "unit": "TOPS", "scaling": "strong",
                    "config": {"workload": f"config3: {L}-layer Q4_K_M stack (q/k/o/gate/up Q4_K, v/down Q6_K) at "
                                           f"M={M}, layers chained through RMSNorm / SwiGLU (attention core outside "
                                           f"the path: o takes q's output)",
                               "m": M, "layers": L, "ops_per_step": ops, "weight_bytes_per_rank": rank_wbytes,
                               "l2": f"inputs larger than L2: {rank_wbytes / 2**20:.0f} MiB of weights per rank",
                               "parallelism": "replicas x1" if world == 1 else
                               f"FFN row-shard x{world} (NCCL all-gathers), projections replicated",
                               "timing": "launches of all layers per step, warm-up steps then timed steps back to "
                                         "back, CUDA events, max over ranks"},
                    "roofline": {"bound": "tensor", "achieved": round(value, 2), "peak": round(peak_int8, 1),
                                 "unit": "TOPS", "frac": round(value / peak_int8, 4),
                                 "peak_source": peak_int8_src, "traffic": None},
                    "e2e": {"value": round(ops * e2e_steps / e2e_dt / 1e12, 2), "unit": "TOPS", "steps": e2e_steps,
                            "h2d_bytes_per_step": M * HIDDEN * 2, "d2h_bytes_per_step": d2h,
                            "api": "pinned input rows copied in, the stack, the last hidden rows copied out"},
                })
            else:
                value = SEQ * steps / dt
                result = dict(common, **{
                    "metric": METRIC_DECODE, "value": round(value, 1), "unit": "tok/s", "scaling": "strong",
                    "config": {"workload": f"config4: {SEQ} sequences x 1 token, {L}-layer stack (q/o/gate/up Q5_K, "
                                           f"k/v/down Q8_0) chained through RMSNorm / SwiGLU + final norm + Q6_K LM head "
                                           f"{VOCAB}x{HIDDEN} vocab-sharded with the argmax merged on the device",
                               "rows_per_rank": M, "layers": L, "weight_bytes_per_step_per_rank": rank_wbytes,
                               "parallelism": f"batch-split x{world}, LM head vocab-split + NCCL all-gathers",
                               "timing": "CUDA graph: warm-up steps, event, timed steps, event; max over ranks"},
                    "roofline": {"bound": "hbm", "achieved": round(rank_wbytes * steps / dt / 1e9, 1), "peak": peak_hbm,
                                 "unit": "GB/s", "frac": round(rank_wbytes * steps / dt / 1e9 / peak_hbm, 4),
                                 "peak_source": peak_kind, "traffic": None},
                    "e2e": {"value": round(SEQ * e2e_steps / e2e_dt, 1), "unit": "tok/s", "steps": e2e_steps,
                            "h2d_bytes_per_step": M * HIDDEN * 2, "d2h_bytes_per_step": d2h,
                            "api": "pinned input rows copied in, the stack + LM head, the 64 next tokens copied out"},
                })
        for lay in layers:
            for w_ in lay.values():
                w_.free()
        if not prefill:
            lm.free()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def ffn_tensor_roofline(tops_per_rank, device):
    """Batched-prefill FFN (hundreds of tokens and more): a dense int8 contraction, so its roofline is
    the tensor-core peak (measured live), per GPU."""
    peak, src = measured_int8_tops(device)
    return {"bound": "tensor", "achieved": round(tops_per_rank, 2), "peak": round(peak, 1), "unit": "TOPS",
            "frac": round(tops_per_rank / peak, 4), "peak_source": src, "traffic": None,
            "note": "int8 TOPS of one rank's share of the block per step time"}


def measured_int8_tops(device):
    """(dense int8 tensor TOPS, how it was obtained): this GPU measured live by kq_measure_int8_tops
    (every SM issuing back-to-back tcgen05.mma kind::i8 128x256x32), else 2 x the measured bf16
    figure."""
    import ctypes as C
    import npu880_mtk_npu_llm_runtime_b200 as kq
    t = C.c_double(0.0)
    try:
        rc = kq.load_library().kq_measure_int8_tops(device, 1024, C.byref(t))
    except (OSError, AttributeError):
        rc = -1
    if rc == 0 and t.value > 0:
        return t.value, ("measured here: kq_measure_int8_tops (tcgen05.mma kind::i8 128x256x32 back to back on "
                         "every SM, s32 in TMEM, best of 3 launches)")
    return 2.0 * measured_bf16(), "assumed: 2 x measured dense bf16 TF/s (the int8 measurement failed)"


def measured_bf16():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


# ---------------------------------------------------------------------------- reference arm

def run_reference(args, rank, world):
    if rank != 0:
        return None
    if args.config not in ("gemv", "lm_head"):
        return {"impl": "reference", "unavailable": "the reference arm times configs 0 and 1; the stack configs carry "
                                                   "their CPU sample in cpu_baseline"}
    from npu880_mtk_npu_llm_runtime_b200 import synth
    gtype = synth.TYPE_Q4_K if args.config == "gemv" else synth.TYPE_Q6_K
    n_rows = 9728 if args.config == "gemv" else 151936
    warmup = max(3, args.warmup)
    # each step is one full GEMV on the reference pool; the step count is capped by time so the
    # whole arm ends within a few minutes
    c = cpu_reference_gemv(n_rows, 2560, gtype, seconds=args.ref_seconds, max_steps=args.steps, warmup=warmup)
    cfg = gemv_config(world) if args.config == "gemv" else lm_config(world)
    if args.config == "lm_head":
        cfg["weight_bytes_per_step_per_rank"] = n_rows * 2100
    v = round(c["value"], 4)
    return {
        "impl": "reference", "metric": METRIC_GEMV if args.config == "gemv" else METRIC_LM,
        "value": v, "unit": "GB/s", "n_gpus": world, "steps": c["steps"], "warmup": warmup,
        "ms_per_step": round(c["seconds_per_step"] * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if args.config == "gemv" else "strong", "vs_baseline": None, "dtype": "int8",
        "data": DATA_DESC, "config": cfg,
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": c["cores"], "kind": c["kind"], "sample": c["sample"],
                         "single_thread": c["single_thread"]},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=STEPS_DEFAULT)
    ap.add_argument("--warmup", type=int, default=300)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["gemv", "lm_head", "ffn", "prefill", "decode"], default="gemv")
    # (not "--m": torchrun's own parser takes it for an abbreviation of its options)
    ap.add_argument("--tokens", "--m", dest="tokens", type=int, default=0, help="tokens (ffn: 8/16/32/64 or 512/2048, prefill: 512/2048)")
    ap.add_argument("--ffn-fused", type=int, default=1, help="ffn: 1 = the persistent FFN kernel where it applies "
                                                              "(1-2 tokens), 0 = the four launches")
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=30.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-lm-head", action="store_true", help="config 0 without the nested sharded LM-head record")
    args = ap.parse_args()
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        res = run_reference(args, rank, world)
    elif args.config in ("ffn", "prefill", "decode"):
        if args.steps == STEPS_DEFAULT:  # the GEMV default is far too many steps for a whole block or stack
            args.steps = {"ffn": 2000, "prefill": 3, "decode": 20}[args.config]
            args.warmup = min(args.warmup, 3)
        res = run_stack(args, rank, world, local_rank)
    else:
        res = run_ours(args, rank, world, local_rank)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
