#!/usr/bin/env python
"""Benchmark of the K-quant x @ W^T hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the Q6_K vocab-head GEMV, M=1, K=2560,
N=151936 -- 319 MB of quantized weights, larger than L2, so every timed step
streams the weights from HBM.  A step is one pass of the hot path: Q8_K
quantization of x then the GEMV.  At N>1 GPUs the rows are sharded N/P per
rank and the fp32 logits are all-gathered over NVLink -- fused into the GEMV
(each rank stores its slice into every peer's buffer and raises a flag there;
default) or by NCCL (--gather nccl); total work is fixed (strong scaling).  Time is measured on the device with CUDA events,
max over ranks.

`--impl reference` times the reference's CPU implementation of the same
workload (the C restatement of its AVX2 kernels under oracle/, all host
threads); under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen3.5sharp_b200"))

METRIC = "K-quant GEMV HBM GB/s (frac of 8 TB/s); M=512 GEMM TFLOP/s; 1/2/4/8 GPU"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CFG = dict(qtype=14, m=1, k=2560, n=151936, seed_w=1, seed_x=2)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return dict(FALLBACK_PEAKS), "fallback"


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.tmp.flush()
        self.tmp.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.tmp.read())) if len(r) >= 9]
        os.unlink(self.tmp.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def traffic_from_profile():
    """Per-launch DRAM bytes of the GEMV kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "gemv_q6k_vocab_m1.txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


def cpu_baseline(w_blocks, x, budget_s: float = 10.0):
    """The reference's CPU GEMV (C restatement of its AVX2 kernels, oracle/)
    on the full workload, with the reference's default worker count
    (CpuTopology.ChooseWorkerCount) and with all host threads."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    from q35k import synth

    oracle.build()
    topo = oracle.host_topology()
    W = oracle.Weight(CFG["qtype"], w_blocks, CFG["k"], w_blocks.shape[0])
    nbytes = synth.algorithmic_bytes(CFG["qtype"], CFG["m"], CFG["k"], w_blocks.shape[0])
    out = {}
    for label, threads in (("reference_workers", topo["reference_workers"]), ("all_threads", topo["logical"])):
        W.matmul(x, threads=threads)  # warm-up (page-in, pool start)
        n, t0 = 0, time.perf_counter()
        while True:
            W.matmul(x, threads=threads)
            n += 1
            el = time.perf_counter() - t0
            if el > budget_s / 2 or n >= 200:
                break
        out[label] = dict(value=nbytes / (el / n) / 1e9, cores=threads, calls=n, seconds=el)
    return out, topo


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    from q35k import synth

    oracle.build()
    topo = oracle.host_topology()
    threads = topo["logical"]
    w = synth.kquant_blocks(CFG["qtype"], CFG["n"], CFG["k"], seed=CFG["seed_w"])
    x = synth.activations(CFG["m"], CFG["k"], seed=CFG["seed_x"])
    W = oracle.Weight(CFG["qtype"], w, CFG["k"], CFG["n"])
    nbytes = synth.algorithmic_bytes(CFG["qtype"], CFG["m"], CFG["k"], CFG["n"])
    for _ in range(args.warmup):
        W.matmul(x, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        W.matmul(x, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = nbytes / (ms / 1e3) / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "cfg1 Q6_K GEMV M=1 K=2560 N=151936 (vocab head)", "qtype": "Q6_K", "m": 1,
                   "k": 2560, "n": 151936, "l2": "inputs > L2 (319 MB of weights)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "full cfg1 GEMV per step (Q8K.QuantizeRow + Q6K.GemvPrequant over all "
                                   "151936 rows), C restatement of the reference's AVX2 kernels, "
                                   f"static row partition over {threads} threads"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host": topo,
    }
    print(json.dumps(line))


def run_ours(args):
    import numpy as np
    import torch

    import q35k
    from q35k import synth

    rank, world, local = dist_env()
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    gather_mode = q35k.GATHER_FUSED if args.gather == "fused" else q35k.GATHER_NCCL
    gather_desc = ("fused into the GEMV (NVLink stores into every peer + bounded flag wait)" if args.gather == "fused"
                   else "NCCL all-gather")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    peaks, peak_kind = load_peaks()
    qt, M, K, N = CFG["qtype"], CFG["m"], CFG["k"], CFG["n"]
    # Rows of this rank: the library's equal-share split (q35k_shard_*).
    r0, r1 = q35k.shard_range(N, world, rank)
    rows = r1 - r0
    w = synth.kquant_blocks(qt, rows, K, seed=CFG["seed_w"], row_start=r0)
    x = synth.activations(M, K, seed=CFG["seed_x"])

    # The rank's own slice on a plain context: the GEMV kernel timed alone
    # (roofline), and the whole step at N = 1.
    ctx = q35k.Context(local)
    W = ctx.upload(qt, w, K, rows)
    # One explicit stream for our kernels, the CUDA events and NCCL.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    dx = torch.from_numpy(x).cuda()
    dy_full = torch.empty((M, N), dtype=torch.float32, device="cuda")
    dy_local = torch.empty((M, rows), dtype=torch.float32, device="cuda")
    group = SW = None
    if world > 1:
        # One process per GPU: rank 0 makes the NCCL id, torch.distributed
        # carries it to the others; the library's group does the rest.
        idt = torch.zeros(q35k._lib.NCCL_ID_BYTES, dtype=torch.uint8, device="cuda")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(q35k.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        group = q35k.Shard(nranks=world, rank=rank, nccl_id=bytes(idt.cpu().numpy().tobytes()), device=local)
        # q35k_shard_weight_upload takes the full matrix and keeps this rank's
        # rows; hand it a view whose rows r0..r1 are this rank's blocks.
        w_view = np.zeros((N, w.shape[1]), dtype=np.uint8)
        w_view[r0:r1] = w
        SW = group.upload(qt, w_view, K, N)
        del w_view

    def step(ev=None):
        # One pass of the hot path: N = 1, q35k_matmul_dev (Q8_K quantization
        # of x fused into the GEMV at M = 1); N > 1, q35k_shard_matmul_dev (the
        # rank's GEMV, then the gather of the logits: fused into the GEMV --
        # NVLink stores into every peer plus a bounded flag wait -- or NCCL's
        # all-gather with --gather nccl).
        if ev:
            ev[0].record(stream)
        if world == 1:
            ctx.matmul_dev(W, dx, dy_full, M, sh)
        else:
            group.matmul_dev(SW, [dx], [dy_full], M, gather_mode, streams=[sh])
        if ev:
            ev[1].record(stream)

    def kernel_only(ev):
        ev[0].record(stream)
        ctx.matmul_dev(W, dx, dy_local, M, sh)
        ev[1].record(stream)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # K steps back to back (nothing between them on the stream, so each
    # step's GEMV may start streaming weights under the previous step's tail,
    # as in a model's decode loop), one event pair around them.
    start.record(stream)
    for i in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = start.elapsed_time(end)
    # Per-step event times, untimed pass (events between steps serialise them).
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    for i in range(args.steps):
        step(evs[i])
    torch.cuda.synchronize()
    step_ms = [e[0].elapsed_time(e[1]) for e in evs]
    # The rank's GEMV kernel timed alone (untimed for the headline).
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    for i in range(args.steps):
        kernel_only(kev[i])
    torch.cuda.synchronize()
    gemv_ms = [e[0].elapsed_time(e[1]) for e in kev]
    ms_step = total_ms / args.steps
    if world > 1:
        t = torch.tensor([ms_step], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())

    nbytes_total = synth.algorithmic_bytes(qt, M, K, N)
    nbytes_local = synth.algorithmic_bytes(qt, M, K, rows)
    value = nbytes_total / (ms_step / 1e3) / 1e9

    # End to end through the public host-pointer API (q35k_matmul): x from
    # host memory, y back to host memory, every step.
    e2e = None
    if world == 1:
        # The caller's output buffer persists across steps, as the reference's
        # model writes through one float* output of its scratch arena.
        y_host = np.empty((M, N), dtype=np.float32)
        for _ in range(3):
            ctx.matmul(W, x, out=y_host)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ctx.matmul(W, x, out=y_host)
        e2e_s = (time.perf_counter() - t0) / args.steps
        e2e = {"value": nbytes_total / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(x.nbytes),
               "d2h_bytes_per_step": int(y_host.nbytes), "ms_per_step": e2e_s * 1e3,
               "api": "q35k_matmul (host pointers, synchronous)"}
    else:
        xh = torch.from_numpy(x).pin_memory()
        yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
        for _ in range(3):
            dx.copy_(xh, non_blocking=True)
            step()
            yh.copy_(dy_full, non_blocking=True)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            dx.copy_(xh, non_blocking=True)
            step()
            yh.copy_(dy_full, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
        e2e = {"value": nbytes_total / (e2e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(x.nbytes),
               "d2h_bytes_per_step": int(M * N * 4), "ms_per_step": e2e_ms,
               "api": f"pinned H2D of x + q35k_shard_matmul_dev (GEMV, gather {gather_desc}) + D2H of y"}

    gemv_avg = sum(gemv_ms) / len(gemv_ms)
    achieved = nbytes_local / (gemv_avg / 1e3) / 1e9
    traffic = traffic_from_profile() if world == 1 else None
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
                "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS,
                "kernel": "q35k_decode_kernel<Q6_K,1,fused>", "kernel_ms": gemv_avg,
                "algorithmic_bytes_per_launch": nbytes_local}

    launches_per_step = count_launches(torch, step)

    extra = {}
    if world == 1 and not args.no_extra:
        extra = secondary_configs(ctx, torch, np, synth, peaks)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        w_full = w  # world == 1: the full matrix
        res, topo = cpu_baseline(w_full, x)
        ref = res["reference_workers"]
        cpu = {"value": ref["value"], "unit": "GB/s", "cores": ref["cores"], "kind": "port",
               "sample": f"{ref['calls']} full cfg1 GEMV calls ({ref['seconds']:.1f} s), C restatement of the "
                         f"reference's AVX2 Q6K.Gemv, reference worker count {ref['cores']}",
               "all_threads": res["all_threads"], "host": topo}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "cfg1 Q6_K GEMV M=1 K=2560 N=151936 (vocab head)", "qtype": "Q6_K", "m": M,
                       "k": K, "n": N, "rows_per_gpu": rows, "l2": "inputs > L2 (319 MB of weights)",
                       "parallelism": (f"row-sharded N/{world}, gather {gather_desc} (q35k_shard_matmul_dev)"
                                       if world > 1 else "single GPU")},
            "frac_of_nominal_8tbs": value / NOMINAL_HBM_GBS,
            "gemv_ms": gemv_avg, "step_ms_events": sum(step_ms) / len(step_ms),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": launches_per_step * args.steps, "launches_per_step": launches_per_step, "also": extra,
        }
        print(json.dumps(line))
    W.free()
    ctx.close()
    if world > 1:
        SW.free()
        group.close()
        dist.barrier()
        dist.destroy_process_group()


OUR_KERNELS = ("q35k_decode_kernel", "quantize_q8k_kernel", "q8k_to_planar_kernel", "dequant_kernel", "repack_tiles_kernel",
               "gemm_prep_kernel", "gemm_q4k_tc_kernel", "gather_permute_kernel", "signal_wait_kernel",
               "argmax_index_kernel", "q4k_meta_kernel", "q6k_meta_kernel")


def count_launches(torch, step):
    """Kernels of libq35k launched by one step, counted with the CUDA
    profiler on an untimed step (NCCL and torch kernels excluded)."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    n = 0
    for ev in prof.events():
        if any(k in ev.name for k in OUR_KERNELS) and ev.device_type.name == "CUDA":
            n += 1
    return n


def secondary_configs(ctx, torch, np, synth, peaks):
    """Device time per call (Q8_K quantize + GEMV, q35k_matmul_dev) for the
    other configs.  They fit in L2, so each timed run cycles through enough
    distinct uploaded copies of the weights to exceed 3x L2 (every launch
    streams cold weights from HBM), and the calls are replayed from a CUDA
    graph so that host launch latency does not enter the device time."""
    out = {}
    stream = torch.cuda.current_stream()
    cases = [("cfg0_q4k_m1", 12, 1, 2560, 9728, 1.0), ("cfg2_q5k_m8", 13, 8, 9728, 2560, 0.5),
             ("cfg4_q4k_m1_p1", 12, 1, 5120, 27648, 1.0), ("cfg4_q4k_m8_p1", 12, 8, 5120, 27648, 1.0)]
    l2 = 126 * 2**20
    for name, qt, m, k, n, scale in cases:
        w = synth.kquant_blocks(qt, n, k, seed=1)
        x = synth.activations(m, k, seed=2, scale=scale)
        copies = max(2, min(64, -(-3 * l2 // w.nbytes)))
        Ws = [ctx.upload(qt, w, k, n) for _ in range(copies)]
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
        for W in Ws:  # warm-up, sizes every scratch buffer before capture
            ctx.matmul_dev(W, dx, dy, m, stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream()
            for W in Ws:
                ctx.matmul_dev(W, dx, dy, m, cs)
        graph.replay()
        torch.cuda.synchronize()
        reps = max(3, 400 // copies)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (reps * copies)
        nbytes = synth.algorithmic_bytes(qt, m, k, n)
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"call_ms": ms, "GB/s": gbs, "frac_measured_hbm": gbs / peaks["hbm_gbs"],
                     "frac_nominal_8tbs": gbs / NOMINAL_HBM_GBS,
                     "timing": f"quantize+GEMV per call, CUDA-graph replay over {copies} weight copies "
                               f"({copies * w.nbytes / 2**20:.0f} MiB > 3x L2)"}
        del graph
        for W in Ws:
            W.free()
    out.update(argmax_config(ctx, torch, synth, peaks))
    out.update(ffn_decode_config(ctx, torch, synth, peaks))
    out.update(gemm_configs(ctx, torch, synth, peaks))
    return out


def ffn_decode_config(ctx, torch, synth, peaks):
    """One decode FFN at cfg0/cfg3's dimensions (hidden 2560, ffn 9728, Q4_K):
    gate and up from one quantization of x in one GEMV launch
    (q35k_matmul_shared_dev), then ffn_down on silu(gate) * up with the
    product formed in its quantization (q35k_matmul_silu_dev); against gate
    and up as two separate calls.  Eight layers' weights (336 MB > L2) cycled
    in a CUDA graph."""
    qt, m, hid, ffn, layers = 12, 1, 2560, 9728, 8
    stream = torch.cuda.current_stream()
    L = []
    for i in range(layers):
        L.append((ctx.upload(qt, synth.kquant_blocks(qt, ffn, hid, seed=3 * i + 1), hid, ffn),
                  ctx.upload(qt, synth.kquant_blocks(qt, ffn, hid, seed=3 * i + 2), hid, ffn),
                  ctx.upload(qt, synth.kquant_blocks(qt, hid, ffn, seed=3 * i + 3), ffn, hid)))
    dx = torch.from_numpy(synth.activations(m, hid, seed=5)).cuda()
    dg = torch.empty((m, ffn), dtype=torch.float32, device="cuda")
    du = torch.empty((m, ffn), dtype=torch.float32, device="cuda")
    dd = torch.empty((m, hid), dtype=torch.float32, device="cuda")

    def shared(cs):
        for g, u, d in L:
            ctx.matmul_shared_dev([g, u], dx, [dg, du], m, cs)
            ctx.matmul_silu_dev(d, dg, du, dd, m, cs)

    def separate(cs):
        for g, u, d in L:
            ctx.matmul_dev(g, dx, dg, m, cs)
            ctx.matmul_dev(u, dx, du, m, cs)
            ctx.matmul_silu_dev(d, dg, du, dd, m, cs)

    res = {}
    nbytes = sum(synth.algorithmic_bytes(qt, m, hid, ffn) for _ in range(2)) + synth.algorithmic_bytes(qt, m, ffn, hid)
    for name, fn in (("shared", shared), ("separate", separate)):
        fn(stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn(torch.cuda.current_stream())
        graph.replay()
        torch.cuda.synchronize()
        reps = 50
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (reps * layers)
        res[name] = (ms, nbytes / (ms / 1e3) / 1e9)
        del graph
    for t in L:
        for W in t:
            W.free()
    ms, gbs = res["shared"]
    return {"cfg3_q4k_m1_ffn_decode": {
        "layer_ms": ms, "GB/s": gbs, "frac_measured_hbm": gbs / peaks["hbm_gbs"],
        "separate_gate_up_layer_ms": res["separate"][0], "separate_GB/s": res["separate"][1],
        "timing": f"gate+up (one shared GEMV launch) + silu-fused ffn_down per layer, CUDA-graph replay over "
                  f"{layers} layers (336 MB of weights > L2)"}}


def argmax_config(ctx, torch, synth, peaks):
    """cfg1's vocab head with the ArgMax fused into the GEMV epilogue
    (q35k_matmul_argmax_dev, logits not written): back-to-back calls on the
    same 319 MB weight (> L2), as a decode loop issues them."""
    qt, m, k, n = 14, 1, 2560, 151936
    w = synth.kquant_blocks(qt, n, k, seed=1)
    x = synth.activations(m, k, seed=2)
    W = ctx.upload(qt, w, k, n)
    dx = torch.from_numpy(x).cuda()
    di = torch.empty(m, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(5):
        ctx.matmul_argmax_dev(W, dx, None, di, m, stream)
    torch.cuda.synchronize()
    reps = 50
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        ctx.matmul_argmax_dev(W, dx, None, di, m, stream)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    nbytes = synth.algorithmic_bytes(qt, m, k, n) - m * n * 4  # no logits written
    gbs = nbytes / (ms / 1e3) / 1e9
    W.free()
    return {"cfg1_q6k_m1_argmax": {"call_ms": ms, "GB/s": gbs, "frac_measured_hbm": gbs / peaks["hbm_gbs"],
                                   "timing": f"{reps} back-to-back q35k_matmul_argmax_dev calls (GEMV + argmax "
                                             f"epilogue + index kernel), CUDA events"}}


def gemm_configs(ctx, torch, synth, peaks):
    """Tensor-core prefill GEMM (Q4_K, M = 512): BASELINE config 3 and config
    4 at M = 512 on one GPU, in both GEMM modes (exact: every product formed
    from the reference's integers, error ~1e-6; fast: fp16-rounded dequantized
    operands, error ~4e-4, within the 1e-3 bar).  Device time per
    q35k_matmul_dev call (Q8_K preparation kernel + GEMM kernel), CUDA-graph
    replay; the weights (14 and 80 MB) sit in L2 after the first call, as in
    any compute-bound GEMM.  TFLOP/s = 2 M N K / time against the measured
    dense bf16 peak."""
    import q35k

    out = {}
    Q4, Q5, Q6 = synth.Q4_K, synth.Q5_K, synth.Q6_K
    # Q5_K / Q6_K at cfg2's ffn_down shape (K = 9728, N = 2560) with GGUF-like
    # scales; Q6_K has no exact tensor-core form (its exact-mode prefill is
    # the GEMV).
    cases = [("cfg3_q4k_gemm_m512", Q4, 512, 2560, 9728), ("cfg4_q4k_gemm_m512_p1", Q4, 512, 5120, 27648),
             ("q5k_gemm_m512_k9728_n2560", Q5, 512, 9728, 2560)]
    for mode, suffix in ((q35k.GEMM_EXACT, ""), (q35k.GEMM_FAST, "_fast")):
        ctx.set_gemm_mode(mode)
        extra = [("q6k_gemm_m512_k9728_n2560", Q6, 512, 9728, 2560)] if mode == q35k.GEMM_FAST else []
        out.update(_gemm_lines(ctx, torch, synth, peaks, suffix, "exact" if mode == q35k.GEMM_EXACT else "fast",
                               cases + extra))
    ctx.set_gemm_mode(q35k.GEMM_EXACT)
    return out


def _gemm_lines(ctx, torch, synth, peaks, suffix, mode_name, cases):
    out = {}
    stream = torch.cuda.current_stream()
    bf16_peak = peaks.get("bf16_tflops")
    for name, qt, m, k, n in cases:
        name = name + suffix
        w = synth.kquant_blocks(qt, n, k, seed=1, q5_uniform_d=False)
        x = synth.activations(m, k, seed=2)
        W = ctx.upload(qt, w, k, n)
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
        for _ in range(3):
            ctx.matmul_dev(W, dx, dy, m, stream)
        torch.cuda.synchronize()
        calls = 10
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream()
            for _ in range(calls):
                ctx.matmul_dev(W, dx, dy, m, cs)
        graph.replay()
        torch.cuda.synchronize()
        reps = 10
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (reps * calls)
        tflops = 2.0 * m * n * k / (ms / 1e3) / 1e12
        out[name] = {"call_ms": ms, "TFLOP/s": tflops, "gemm_mode": mode_name,
                     "frac_measured_bf16": (tflops / bf16_peak) if bf16_peak else None,
                     "peak_kind": "measured dense bf16 (MEASURED_PEAKS.json bf16_tflops)",
                     "kernels": "gemm_prep_kernel + gemm_q4k_tc_kernel (tcgen05, TMEM, TMA)",
                     "timing": f"CUDA-graph replay of {calls} calls x {reps}"}
        del graph
        W.free()
    return out


# Configurations runnable alone under a profiler: (qtype, M, K, N, x scale,
# GEMM mode).
PROFILE_CASES = {
    "cfg0_q4k_m1": (12, 1, 2560, 9728, 1.0, 0),
    "cfg1_q6k_m1": (14, 1, 2560, 151936, 1.0, 0),
    "cfg2_q5k_m8": (13, 8, 9728, 2560, 0.5, 0),
    "cfg3_q4k_gemm_m512": (12, 512, 2560, 9728, 1.0, 0),
    "cfg3_q4k_gemm_m512_fast": (12, 512, 2560, 9728, 1.0, 1),
    "cfg3_q4k_gemm_m64": (12, 64, 2560, 9728, 1.0, 0),
    "cfg4_q4k_m1_p1": (12, 1, 5120, 27648, 1.0, 0),
    "cfg4_q4k_m8_p1": (12, 8, 5120, 27648, 1.0, 0),
    "cfg4_q4k_gemm_m512_p1": (12, 512, 5120, 27648, 1.0, 0),
    "cfg4_q4k_gemm_m512_p1_fast": (12, 512, 5120, 27648, 1.0, 1),
    "q5k_gemm_m512": (13, 512, 9728, 2560, 1.0, 0),
    "q5k_gemm_m512_fast": (13, 512, 9728, 2560, 1.0, 1),
    "q6k_gemm_m512_fast": (14, 512, 9728, 2560, 1.0, 1),
}


def run_profile_case(args):
    """Upload one configuration's weight and run --steps q35k_matmul_dev
    calls (device pointers, the context's stream), then synchronize: a small,
    self-contained command for ncu captures."""
    import torch

    import q35k
    from q35k import synth

    qt, m, k, n, scale, mode = PROFILE_CASES[args.profile]
    ctx = q35k.Context(0)
    ctx.set_gemm_mode(mode)
    # GEMM cases: GGUF-like Q5_K scales (the fast mode's fp16 weights need them)
    W = ctx.upload(qt, synth.kquant_blocks(qt, n, k, seed=1, q5_uniform_d=m < 16), k, n)
    dx = torch.from_numpy(synth.activations(m, k, seed=2, scale=scale)).cuda()
    dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
    for _ in range(args.steps):
        ctx.matmul_dev(W, dx, dy, m, None)
    ctx.sync()
    W.free()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary configs")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="N > 1: how the ranks' output slices are all-gathered")
    ap.add_argument("--profile", choices=sorted(PROFILE_CASES),
                    help="only run --steps q35k_matmul_dev calls of one configuration (for ncu), no timing output")
    args = ap.parse_args()
    if args.profile:
        run_profile_case(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
