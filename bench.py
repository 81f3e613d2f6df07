#!/usr/bin/env python
"""Benchmark of the K-quant x @ W^T hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: the Q6_K vocab-head GEMV, M=1,
K=2560, N=151936 -- 319 MB of quantized weights, larger than L2, so every
timed step streams the weights from HBM.  A step is one pass of the hot path:
Q8_K quantization of x then the GEMV.  At N>1 GPUs the rows are sharded N/P
per rank and the fp32 logits are all-gathered over NVLink -- fused into the
GEMV (each rank stores its slice into every peer's buffer and raises a flag
there; default) or by NCCL (--gather nccl); total work is fixed (strong
scaling).  Time is measured on the device with CUDA events, max over ranks.

Every other configuration of BASELINE.json is measured too and reported in
`roofline["configs"]` (value, fraction of the measured peak, parity) and, at
N = 1, `cpu_baseline["configs"]` (the reference's CPU kernels on the same
inputs): cfg0, cfg2 and cfg4 at M = 1 / 8 (decode GEMV), cfg3 and cfg4 at
M = 512 (tensor-core GEMM, both arithmetic modes), and at N > 1 the sharded
cfg4 at M = 1, 8, 512 with its gather.  The same figures are printed as short
`# cfg` lines before the headline JSON line.

`--impl reference` times the reference's CPU implementation of the headline
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
# The headline config, identical in both arms' JSON lines.
CONFIG = {"workload": "cfg1 Q6_K GEMV M=1 K=2560 N=151936 (vocab head)", "qtype": "Q6_K", "m": 1, "k": 2560,
          "n": 151936, "l2": "inputs > L2 (319 MB of weights)"}
Q4, Q5, Q6 = 12, 13, 14
TYPE_NAME = {Q4: "Q4_K", Q5: "Q5_K", Q6: "Q6_K"}
# Secondary decode configurations (cold weights): name, type, M, K, N, x scale.
GEMV_CASES = [("cfg0", Q4, 1, 2560, 9728, 1.0), ("cfg2", Q5, 8, 9728, 2560, 0.5),
              ("cfg4_m1", Q4, 1, 5120, 27648, 1.0), ("cfg4_m8", Q4, 8, 5120, 27648, 1.0)]
# Prefill GEMM configurations: name, type, M, K, N.  Q5_K / Q6_K at cfg2's
# ffn_down shape with GGUF-like scales.
GEMM_CASES = [("cfg3", Q4, 512, 2560, 9728), ("cfg4_m512", Q4, 512, 5120, 27648),
              ("q5k_m512", Q5, 512, 9728, 2560), ("q6k_m512", Q6, 512, 9728, 2560)]
# Sharded configuration 4 at every N: name, M (K = 5120, N = 27648, Q4_K).
SHARD_CASES = [("cfg4_m1", 1), ("cfg4_m8", 8), ("cfg4_m512", 512)]
CFG4_K, CFG4_N = 5120, 27648
OUR_KERNELS = ("q35k_decode_kernel", "quantize_q8k_kernel", "q8k_to_planar_kernel", "dequant_kernel",
               "repack_tiles_kernel", "gemm_prep_kernel", "gemm_q4k_tc_kernel", "gather_permute_kernel",
               "q35k_shard_gather_kernel", "argmax_index_kernel", "q4k_meta_kernel", "q6k_meta_kernel",
               "q35k_stage_in_kernel", "q35k_err_out_kernel", "gemm_prep_fast_kernel", "gemm_token_max_kernel",
               "fast_row_scale_kernel", "q4k_fast_meta_kernel", "q6k_fast_meta_kernel")


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
    """Per-launch DRAM bytes of the headline GEMV from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "gemv_q6k_vocab_m1.txt")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


def rel_err(y, r) -> float:
    import numpy as np

    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    return float(np.abs(y - r).max() / max(float(np.abs(r).max()), 1e-30))


def elem_rel_err(y, r) -> float:
    """Largest element-wise |y - r| / |r| over the outputs with |r| >= 1e-2
    max |r| (the second parity figure, beside rel_err)."""
    import numpy as np

    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(r, dtype=np.float64)
    big = np.abs(r) >= 1e-2 * max(float(np.abs(r).max()), 1e-30)
    return float((np.abs(y - r)[big] / np.abs(r)[big]).max()) if big.any() else 0.0


def count_launches(torch, step):
    """Kernels of libq35k launched by one step, counted with the CUDA
    profiler on an untimed step (NCCL and torch kernels excluded)."""
    return len(kernels_of(torch, step))


def kernels_of(torch, step):
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    return [ev.name for ev in prof.events()
            if any(k in ev.name for k in OUR_KERNELS) and ev.device_type.name == "CUDA"]


# ---------------------------------------------------------------------------
# CPU leg: the reference's kernels (the oracle's C restatement) on the box's
# host cores, timed as the CPU baseline, and used as the checker of the GPU
# outputs the GPU legs kept.
# ---------------------------------------------------------------------------

def cpu_leg(jobs, time_it: bool, budget_s: float = 1.0):
    """jobs: name -> (qtype, blocks, x, gpu_y, rows) where `rows` (None: all)
    selects the output rows compared; only whole-matrix jobs are timed.
    Returns (per-config results, host topology)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle
    from q35k import synth

    oracle.build()
    topo = oracle.host_topology()
    workers = topo["reference_workers"]
    out = {}
    for name, (qt, w, x, gy, rows) in jobs.items():
        m, k = x.shape
        n = w.shape[0]
        res = {}
        if rows is not None:
            W = oracle.Weight(qt, np.ascontiguousarray(w[rows]), k, len(rows))
            ref = W.matmul(x, threads=topo["logical"])
            res["err"], res["err_elem"] = rel_err(gy[:, rows], ref), elem_rel_err(gy[:, rows], ref)
            out[name] = res
            continue
        W = oracle.Weight(qt, w, k, n)
        ref = W.matmul(x, threads=topo["logical"])
        res["err"], res["err_elem"] = rel_err(gy, ref), elem_rel_err(gy, ref)
        if time_it:
            W.matmul(x, threads=workers)  # warm-up
            calls, t0 = 0, time.perf_counter()
            while True:
                W.matmul(x, threads=workers)
                calls += 1
                el = time.perf_counter() - t0
                if el > budget_s or calls >= 200:
                    break
            s = el / calls
            if m >= 64:
                res.update(value=2.0 * m * n * k / s / 1e12, unit="TFLOP/s")
            else:
                res.update(value=synth.algorithmic_bytes(qt, m, k, n) / s / 1e9, unit="GB/s")
            res.update(cores=workers, calls=calls, seconds=el)
        out[name] = res
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
        "config": dict(CONFIG),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "full cfg1 GEMV per step (Q8K.QuantizeRow + Q6K.GemvPrequant over all "
                                   "151936 rows), C restatement of the reference's AVX2 kernels, "
                                   f"static row partition over {threads} threads"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host": topo,
    }
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# GPU legs.
# ---------------------------------------------------------------------------

class Bench:
    def __init__(self, args):
        import numpy as np
        import torch

        import q35k
        from q35k import synth

        self.args, self.np, self.torch, self.q35k, self.synth = args, np, torch, q35k, synth
        self.rank, self.world, self.local = dist_env()
        assert self.world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={self.world}"
        torch.cuda.set_device(self.local)
        self.dist = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        self.peaks, self.peak_kind = load_peaks()
        self.ctx = q35k.Context(self.local)
        self.stream = torch.cuda.Stream()
        torch.cuda.set_stream(self.stream)
        self.sh = self.stream.cuda_stream
        self.group = None
        if self.world > 1:
            # One process per GPU: rank 0 makes the NCCL id, torch.distributed
            # carries it to the others; the library's group does the rest.
            idt = torch.zeros(q35k._lib.NCCL_ID_BYTES, dtype=torch.uint8, device="cuda")
            if self.rank == 0:
                idt.copy_(torch.frombuffer(bytearray(q35k.nccl_unique_id()), dtype=torch.uint8))
            self.dist.broadcast(idt, 0)
            self.group = q35k.Shard(nranks=self.world, rank=self.rank, nccl_id=bytes(idt.cpu().numpy().tobytes()),
                                    device=self.local)
        self.gather_mode = q35k.GATHER_FUSED if args.gather == "fused" else q35k.GATHER_NCCL
        self.gather_desc = ("fused into the GEMV (NVLink stores into every peer + bounded flag wait)"
                            if args.gather == "fused" else "NCCL all-gather")
        self.cpu_jobs = {}   # name -> inputs and GPU output for the CPU leg
        self.configs = {}    # name -> per-config result

    # -- helpers --
    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def event_pair(self):
        return (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))

    def back_to_back_ms(self, fn, steps: int) -> float:
        """ms per call of `steps` calls issued back to back between one event
        pair (max over ranks)."""
        torch = self.torch
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        a, b = self.event_pair()
        a.record(self.stream)
        for _ in range(steps):
            fn()
        b.record(self.stream)
        torch.cuda.synchronize()
        return self.max_over_ranks(a.elapsed_time(b) / steps)

    def graph_ms(self, issue, calls_per_replay, reps):
        """ms per call of a CUDA graph of `calls_per_replay` calls replayed
        `reps` times."""
        torch = self.torch
        issue(self.stream)  # warm-up, sizes every scratch buffer before capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            issue(torch.cuda.current_stream())
        graph.replay()
        torch.cuda.synchronize()
        a, b = self.event_pair()
        a.record(self.stream)
        for _ in range(reps):
            graph.replay()
        b.record(self.stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / (reps * calls_per_replay)
        del graph
        return ms

    def sharded_weight(self, qt, w_rows, k, n, r0, r1):
        """q35k_shard_weight_upload takes the full matrix and keeps this rank's
        rows; hand it a view whose rows r0..r1 are this rank's blocks."""
        np = self.np
        full = np.zeros((n, w_rows.shape[1]), dtype=np.uint8)
        full[r0:r1] = w_rows
        return self.group.upload(qt, full, k, n)

    def boundary_rows(self, n):
        """First and last 64 rows of every rank's slice."""
        rows = []
        for r in range(self.world):
            a, b = self.q35k.shard_range(n, self.world, r)
            rows += list(range(a, min(b, a + 64))) + list(range(max(a, b - 64), b))
        return sorted(set(rows))

    def parity_vs_single_gpu(self, qt, k, n, x, y_mine, make_full, w_local, r0, r1):
        """Rank 0 runs the full matrix on its GPU alone (q35k_matmul_dev) and
        broadcasts y; every rank compares its gathered y with it.  Returns the
        largest relative difference over the ranks and whether every rank's y
        has the same bits (the full matrix alone may take another launch plan
        than a rank's rows, so its fp32 summation order may differ).  Also
        whether the gather is lossless: each rank's own rows computed by one
        plain call on its GPU equal its slice of the gathered y bit for bit,
        and every rank gathered the same bits (a checksum compared across the
        ranks)."""
        np, torch = self.np, self.torch
        m = x.shape[0]
        Wl = self.ctx.upload(qt, w_local, k, r1 - r0)
        alone = torch.empty((m, r1 - r0), dtype=torch.float32, device="cuda")
        self.ctx.matmul_dev(Wl, torch.from_numpy(x).cuda(), alone, m, self.sh)
        torch.cuda.synchronize()
        Wl.free()
        slice_ok = np.array_equal(alone.cpu().numpy().view(np.uint32),
                                  np.ascontiguousarray(y_mine[:, r0:r1]).view(np.uint32))
        bits = y_mine.view(np.uint32).astype(np.uint64).reshape(-1)
        cs = int((bits * (np.arange(bits.size, dtype=np.uint64) | np.uint64(1))).sum() & np.uint64(2**62 - 1))
        cmp = torch.tensor([cs, -cs, 0 if slice_ok else 1], device="cuda", dtype=torch.int64)
        self.dist.all_reduce(cmp, op=self.dist.ReduceOp.MAX)
        lossless = bool(cmp[0].item() == -cmp[1].item() and cmp[2].item() == 0)
        ref = torch.empty((m, n), dtype=torch.float32, device="cuda")
        if self.rank == 0:
            wf = make_full()
            Wf = self.ctx.upload(qt, wf, k, n)
            self.ctx.matmul_dev(Wf, torch.from_numpy(x).cuda(), ref, m, self.sh)
            torch.cuda.synchronize()
            Wf.free()
            del wf
        torch.cuda.synchronize()
        self.dist.broadcast(ref, 0)
        torch.cuda.synchronize()
        r = ref.cpu().numpy()
        err = rel_err(y_mine, r)
        differ = 0.0 if np.array_equal(y_mine.view(np.uint32), r.view(np.uint32)) else 1.0
        t = torch.tensor([err, differ], device="cuda", dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return {"max_rel_err_vs_1gpu": float(t[0].item()), "bit_equal_1gpu": bool(t[1].item() == 0.0),
                "gather_bit_exact": lossless}

    # -- the headline: cfg1 vocab head --
    def headline(self):
        torch, q35k, synth, args = self.torch, self.q35k, self.synth, self.args
        world, rank = self.world, self.rank
        qt, M, K, N = CFG["qtype"], CFG["m"], CFG["k"], CFG["n"]
        r0, r1 = q35k.shard_range(N, world, rank)
        rows = r1 - r0
        w = synth.kquant_blocks(qt, rows, K, seed=CFG["seed_w"], row_start=r0)
        x = synth.activations(M, K, seed=CFG["seed_x"])
        W = self.ctx.upload(qt, w, K, rows)
        dx = torch.from_numpy(x).cuda()
        dy_full = torch.empty((M, N), dtype=torch.float32, device="cuda")
        dy_local = torch.empty((M, rows), dtype=torch.float32, device="cuda")
        SW = self.sharded_weight(qt, w, K, N, r0, r1) if world > 1 else None
        ctx, sh = self.ctx, self.sh

        def step(stream_handle=None):
            # One pass of the hot path: N = 1, q35k_matmul_dev (Q8_K quantization
            # of x fused into the GEMV at M = 1); N > 1, q35k_shard_matmul_dev (the
            # rank's GEMV, then the gather of the logits).
            st = sh if stream_handle is None else stream_handle
            if world == 1:
                ctx.matmul_dev(W, dx, dy_full, M, st)
            else:
                self.group.matmul_dev(SW, [dx], [dy_full], M, self.gather_mode, streams=[st])

        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        self.barrier()
        # The K timed steps are issued from a CUDA graph captured once (a
        # decode loop is launch-bound at 8 GPUs, where a step's device time
        # falls below the host's time to issue it; every call's kernel
        # arguments are the same from call to call, so the call can be
        # captured).  The same steps issued as plain launches are reported
        # beside it.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream().cuda_stream
            for _ in range(args.steps):
                step(cs)
        graph.replay()
        torch.cuda.synchronize()
        self.barrier()
        clocks = ClockSampler(self.local)
        clocks.start()
        ms_step = self.back_to_back_ms(graph.replay, 1) / args.steps
        clk = clocks.stop()
        extra = {"timing": f"{args.steps} steps replayed from one CUDA graph between one pair of CUDA events, "
                           "max over ranks"}
        extra["ms_per_step_launches"] = self.back_to_back_ms(step, args.steps)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        extra["host_issue_ms_per_step"] = (time.perf_counter() - t0) / args.steps * 1e3
        torch.cuda.synchronize()
        self.barrier()
        del graph
        if world > 1:
            # Phase breakdown of one isolated call on this rank's GPU.
            self.barrier()
            self.group.set_trace(True)
            step()
            torch.cuda.synchronize()
            tr = self.group.trace(0)
            self.group.set_trace(False)
            us = lambda a, b: (tr[b] - tr[a]) / 1e3  # noqa: E731
            extra["phases_us"] = {"gemv": us("gemv_start", "gemv_end"),
                                  "gather_start_after_gemv_start": us("gemv_start", "gather_start"),
                                  "peers_seen_after_gemv_end": us("gemv_end", "peers_seen"),
                                  "gemv_done_seen_after_gemv_end": us("gemv_end", "gemv_done_seen"),
                                  "total": us("gemv_start", "gather_end")}
        # Per-step event times (untimed pass: events between steps serialise them).
        evs = [self.event_pair() for _ in range(args.steps)]
        self.barrier()
        for e in evs:
            e[0].record(self.stream)
            step()
            e[1].record(self.stream)
        torch.cuda.synchronize()
        step_ms = [e[0].elapsed_time(e[1]) for e in evs]
        # The rank's GEMV kernel alone (the roofline's kernel): its average
        # launch duration over K launches replayed from a CUDA graph, as the
        # timed steps are (at N = 1 a step is exactly this one kernel), and a
        # single launch between its own pair of events (launch latency included).
        ctx.matmul_dev(W, dx, dy_local, M, self.sh)  # sizes this call's scratch before the capture
        torch.cuda.synchronize()
        kgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kgraph):
            cs = torch.cuda.current_stream().cuda_stream
            for _ in range(args.steps):
                ctx.matmul_dev(W, dx, dy_local, M, cs)
        kgraph.replay()
        torch.cuda.synchronize()
        a_ev, b_ev = self.event_pair()
        a_ev.record(self.stream)
        kgraph.replay()
        b_ev.record(self.stream)
        torch.cuda.synchronize()
        gemv_ms = a_ev.elapsed_time(b_ev) / args.steps
        del kgraph
        kev = [self.event_pair() for _ in range(args.steps)]
        for e in kev:
            e[0].record(self.stream)
            ctx.matmul_dev(W, dx, dy_local, M, sh)
            e[1].record(self.stream)
        torch.cuda.synchronize()
        extra["kernel_ms_isolated"] = sum(e[0].elapsed_time(e[1]) for e in kev) / len(kev)

        nbytes_total = synth.algorithmic_bytes(qt, M, K, N)
        nbytes_local = synth.algorithmic_bytes(qt, M, K, rows)
        value = nbytes_total / (ms_step / 1e3) / 1e9
        launches = count_launches(torch, step)

        # Parity of the gathered logits: at N > 1 against the single-GPU result
        # of the full matrix on every rank; on rank 0 against the oracle (the
        # whole matrix at N = 1, the rows around every shard boundary at N > 1).
        step()
        torch.cuda.synchronize()
        y_mine = dy_full.cpu().numpy()
        self.head_parity = {}
        if world > 1:
            self.head_parity = self.parity_vs_single_gpu(
                qt, K, N, x, y_mine, lambda: synth.kquant_blocks(qt, N, K, seed=CFG["seed_w"]), w, r0, r1)
        if rank == 0:
            self.cpu_jobs["cfg1"] = (qt, w if world == 1 else None, x, y_mine,
                                     None if world == 1 else self.boundary_rows(N))

        e2e = self.e2e(W, x, dx, dy_full, step, nbytes_total)
        achieved = nbytes_local / (gemv_ms / 1e3) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": self.peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": achieved / self.peaks["hbm_gbs"], "traffic": traffic_from_profile() if world == 1 else None,
                    "peak_kind": (f"{self.peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if self.peak_kind == "measured"
                                  else "fallback"),
                    "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS,
                    "kernel": "q35k_decode_kernel_10w<Q6_K,1,fused>", "kernel_ms": gemv_ms,
                    "kernel_timing": f"average of {args.steps} launches replayed from one CUDA graph, CUDA events "
                                     "on the launching stream",
                    "algorithmic_bytes_per_launch": nbytes_local}
        self.head = dict(value=value, ms_step=ms_step, step_ms=sum(step_ms) / len(step_ms), gemv_ms=gemv_ms,
                         rows=rows, clocks=clk, launches=launches, roofline=roofline, e2e=e2e, extra=extra)
        self.head_w = (W, SW)

    def e2e(self, W, x, dx, dy_full, step, nbytes_total):
        """The same metric end to end through the public API: x from host
        memory and y back to host memory every step."""
        np, torch, args = self.np, self.torch, self.args
        M, N = x.shape[0], dy_full.shape[1]
        if self.world == 1:
            # The caller's input and output buffers persist across steps (the
            # reference model's NativeBuffers) and are registered once with
            # q35k_host_register, so q35k_matmul reads x and writes y in place.
            x_host = self.q35k.page_aligned_empty(x.shape)
            y_host = self.q35k.page_aligned_empty((M, N))
            x_host[...] = x
            self.ctx.host_register(x_host)
            self.ctx.host_register(y_host)
            try:
                for _ in range(3):
                    self.ctx.matmul(W, x_host, out=y_host)
                t0 = time.perf_counter()
                for _ in range(args.steps):
                    self.ctx.matmul(W, x_host, out=y_host)
                s = (time.perf_counter() - t0) / args.steps
            finally:
                self.ctx.host_unregister(x_host)
                self.ctx.host_unregister(y_host)
            # The same with pageable buffers (staged through the context).
            y_page = np.empty((M, N), dtype=np.float32)
            for _ in range(3):
                self.ctx.matmul(W, x, out=y_page)
            t0 = time.perf_counter()
            for _ in range(args.steps):
                self.ctx.matmul(W, x, out=y_page)
            s_page = (time.perf_counter() - t0) / args.steps
            return {"value": nbytes_total / s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(x.nbytes),
                    "d2h_bytes_per_step": int(M * N * 4), "ms_per_step": s * 1e3,
                    "api": "q35k_matmul (host pointers, synchronous; x and y registered with q35k_host_register)",
                    "pageable_ms_per_step": s_page * 1e3}
        xh = torch.from_numpy(x).pin_memory()
        yh = torch.empty((M, N), dtype=torch.float32).pin_memory()

        def e2e_step():
            dx.copy_(xh, non_blocking=True)
            step()
            yh.copy_(dy_full, non_blocking=True)

        for _ in range(3):
            e2e_step()
        ms = self.back_to_back_ms(e2e_step, args.steps)
        return {"value": nbytes_total / (ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(x.nbytes),
                "d2h_bytes_per_step": int(M * N * 4), "ms_per_step": ms,
                "api": f"pinned H2D of x + q35k_shard_matmul_dev (GEMV, gather {self.gather_desc}) + D2H of y"}

    # -- secondary configurations at N = 1 --
    def gemv_configs(self):
        """Device time per call (Q8_K quantize + GEMV, q35k_matmul_dev).  These
        weights fit in L2, so each timed run cycles through enough distinct
        uploaded copies to exceed 3x L2 (every launch streams cold weights from
        HBM), replayed from a CUDA graph so host launch latency is not in the
        device time."""
        torch, synth = self.torch, self.synth
        l2 = 126 * 2**20
        for name, qt, m, k, n, scale in GEMV_CASES:
            w = synth.kquant_blocks(qt, n, k, seed=1)
            x = synth.activations(m, k, seed=2, scale=scale)
            copies = max(2, min(64, -(-3 * l2 // w.nbytes)))
            Ws = [self.ctx.upload(qt, w, k, n) for _ in range(copies)]
            dx = torch.from_numpy(x).cuda()
            dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
            ms = self.graph_ms(lambda cs: [self.ctx.matmul_dev(W, dx, dy, m, cs) for W in Ws], copies,
                               max(3, 400 // copies))
            gbs = synth.algorithmic_bytes(qt, m, k, n) / (ms / 1e3) / 1e9
            self.configs[name] = {"v": gbs, "u": "GB/s", "frac": gbs / self.peaks["hbm_gbs"], "ms": ms,
                                  "what": f"{TYPE_NAME[qt]} M={m} K={k} N={n} GEMV, cold weights"}
            torch.cuda.synchronize()
            self.cpu_jobs[name] = (qt, w, x, dy.cpu().numpy(), None)
            for W in Ws:
                W.free()

    def gemm_configs(self):
        """Tensor-core prefill GEMM at M = 512 in both arithmetic modes (exact:
        the reference's integer products, the default; fast: fp16-rounded
        dequantized operands).  Device time per q35k_matmul_dev call (Q8_K
        preparation + GEMM), CUDA-graph replay; the weights sit in L2 after the
        first call, as in any compute-bound GEMM.  TFLOP/s = 2 M N K / time."""
        torch, synth, q35k = self.torch, self.synth, self.q35k
        peak = self.peaks.get("bf16_tflops")
        for name, qt, m, k, n in GEMM_CASES:
            w = synth.kquant_blocks(qt, n, k, seed=1, q5_uniform_d=False)
            x = synth.activations(m, k, seed=2)
            W = self.ctx.upload(qt, w, k, n)
            dx = torch.from_numpy(x).cuda()
            dy = torch.empty((m, n), dtype=torch.float32, device="cuda")
            for mode, suffix in ((q35k.GEMM_EXACT, "_exact"), (q35k.GEMM_FAST, "_fast")):
                self.ctx.set_gemm_mode(mode)
                calls = 10
                ms = self.graph_ms(lambda cs: [self.ctx.matmul_dev(W, dx, dy, m, cs) for _ in range(calls)], calls, 10)
                tf = 2.0 * m * n * k / (ms / 1e3) / 1e12
                names = kernels_of(torch, lambda: self.ctx.matmul_dev(W, dx, dy, m, self.sh))
                path = "tcgen05 GEMM" if any("gemm_q4k_tc_kernel" in s for s in names) else "decode GEMV chunks"
                self.configs[name + suffix] = {"v": tf, "u": "TFLOP/s", "frac": tf / peak if peak else None, "ms": ms,
                                               "what": f"{TYPE_NAME[qt]} M={m} K={k} N={n} {path}"}
                # Checked against the oracle: exact mode on the whole matrix
                # (timed there as the CPU baseline), fast mode on a row subset.
                torch.cuda.synchronize()
                y = dy.cpu().numpy()
                rows = None if mode == q35k.GEMM_EXACT else list(range(0, n, max(1, n // 256)))
                self.cpu_jobs[name + suffix] = (qt, w, x, y, rows)
            self.ctx.set_gemm_mode(q35k.GEMM_EXACT)
            W.free()

    def argmax_config(self):
        """cfg1's vocab head with ArgMax fused into the GEMV epilogue
        (q35k_matmul_argmax_dev, logits not written), back to back."""
        torch, synth = self.torch, self.synth
        W = self.head_w[0]
        qt, m, k, n = CFG["qtype"], CFG["m"], CFG["k"], CFG["n"]
        dx = torch.from_numpy(synth.activations(m, k, seed=CFG["seed_x"])).cuda()
        di = torch.empty(m, dtype=torch.int32, device="cuda")
        for _ in range(5):
            self.ctx.matmul_argmax_dev(W, dx, None, di, m, self.sh)
        ms = self.back_to_back_ms(lambda: self.ctx.matmul_argmax_dev(W, dx, None, di, m, self.sh), 50)
        gbs = (synth.algorithmic_bytes(qt, m, k, n) - m * n * 4) / (ms / 1e3) / 1e9
        self.configs["cfg1_argmax"] = {"v": gbs, "u": "GB/s", "frac": gbs / self.peaks["hbm_gbs"], "ms": ms,
                                       "what": "Q6_K vocab head + fused ArgMax, no logits written"}

    def ffn_config(self):
        """One decode FFN at cfg3's dimensions (hidden 2560, ffn 9728, Q4_K):
        gate and up from one quantization of x in one GEMV launch, then
        ffn_down on silu(gate) * up with the product formed in its
        quantization.  Eight layers' weights (336 MB > L2) in a CUDA graph."""
        torch, synth = self.torch, self.synth
        qt, m, hid, ffn, layers = Q4, 1, 2560, 9728, 8
        L = []
        for i in range(layers):
            L.append((self.ctx.upload(qt, synth.kquant_blocks(qt, ffn, hid, seed=3 * i + 1), hid, ffn),
                      self.ctx.upload(qt, synth.kquant_blocks(qt, ffn, hid, seed=3 * i + 2), hid, ffn),
                      self.ctx.upload(qt, synth.kquant_blocks(qt, hid, ffn, seed=3 * i + 3), ffn, hid)))
        dx = torch.from_numpy(synth.activations(m, hid, seed=5)).cuda()
        dg = torch.empty((m, ffn), dtype=torch.float32, device="cuda")
        du = torch.empty((m, ffn), dtype=torch.float32, device="cuda")
        dd = torch.empty((m, hid), dtype=torch.float32, device="cuda")

        def layers_fn(cs):
            for g, u, d in L:
                self.ctx.matmul_shared_dev([g, u], dx, [dg, du], m, cs)
                self.ctx.matmul_silu_dev(d, dg, du, dd, m, cs)

        ms = self.graph_ms(layers_fn, layers, 50)
        nbytes = 2 * synth.algorithmic_bytes(qt, m, hid, ffn) + synth.algorithmic_bytes(qt, m, ffn, hid)
        gbs = nbytes / (ms / 1e3) / 1e9
        self.configs["ffn_decode"] = {"v": gbs, "u": "GB/s", "frac": gbs / self.peaks["hbm_gbs"], "ms": ms,
                                      "what": "Q4_K gate+up (one shared launch) + SiLU-fused down, M=1, per layer"}
        for t in L:
            for W in t:
                W.free()

    # -- the sharded configuration 4 at N > 1 --
    def shard_configs(self):
        """cfg4 (Q4_K, K=5120, N=27648) row-sharded over the N GPUs at M = 1,
        8 (decode GEMV, gather fused into it) and 512 (tensor-core GEMM, then
        NCCL's all-gather and a permute): device time per call issued back to
        back, max over ranks; the gathered y checked on every rank against
        rank 0's single-GPU result, and on rank 0 against the oracle on the
        rows around every shard boundary."""
        torch, synth, q35k = self.torch, self.synth, self.q35k
        qt, k, n = Q4, CFG4_K, CFG4_N
        r0, r1 = q35k.shard_range(n, self.world, self.rank)
        w = synth.kquant_blocks(qt, r1 - r0, k, seed=1, row_start=r0)
        SW = self.sharded_weight(qt, w, k, n, r0, r1)
        peak_bf16 = self.peaks.get("bf16_tflops")
        for name, m in SHARD_CASES:
            x = synth.activations(m, k, seed=2)
            dx = torch.from_numpy(x).cuda()
            dy = torch.empty((m, n), dtype=torch.float32, device="cuda")

            def call():
                self.group.matmul_dev(SW, [dx], [dy], m, self.gather_mode, streams=[self.sh])

            for _ in range(3):
                call()
            if m <= 8:
                # Decode calls (fused gather): replayed from a CUDA graph, as the
                # headline steps are.
                torch.cuda.synchronize()
                self.barrier()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    cs = torch.cuda.current_stream().cuda_stream
                    for _ in range(20):
                        self.group.matmul_dev(SW, [dx], [dy], m, self.gather_mode, streams=[cs])
                graph.replay()
                torch.cuda.synchronize()
                ms = self.back_to_back_ms(graph.replay, 1) / 20
                del graph
            else:
                ms = self.back_to_back_ms(call, 10)
            call()
            torch.cuda.synchronize()
            y = dy.cpu().numpy()
            par = self.parity_vs_single_gpu(qt, k, n, x, y, lambda: synth.kquant_blocks(qt, n, k, seed=1), w, r0, r1)
            if m >= 64:
                v, u = 2.0 * m * n * k / (ms / 1e3) / 1e12, "TFLOP/s"
                frac = v / peak_bf16 if peak_bf16 else None
                gather = "NCCL all-gather + permute"
            else:
                v, u = synth.algorithmic_bytes(qt, m, k, n) / (ms / 1e3) / 1e9, "GB/s"
                frac = v / self.peaks["hbm_gbs"]
                gather = "gather fused into the GEMV" if self.gather_mode == q35k.GATHER_FUSED else "NCCL all-gather"
            self.configs[f"{name}_p{self.world}"] = {
                "v": v, "u": u, "frac_per_gpu": frac / self.world if frac is not None else None, "ms": ms,
                "err_1gpu": par["max_rel_err_vs_1gpu"], "bit_eq_1gpu": par["bit_equal_1gpu"],
                "gather_exact": par["gather_bit_exact"],
                "what": f"Q4_K M={m} K={k} N={n} row-sharded over {self.world} GPUs, {gather}, whole job"}
            if self.rank == 0:
                self.cpu_jobs[f"{name}_p{self.world}"] = (qt, None, x, y, self.boundary_rows(n))
        SW.free()

    def cpu_checks(self):
        """The CPU leg: at N = 1 the reference's kernels timed on every config
        (the CPU baseline) and checked against the GPU outputs; at N > 1 the
        gathered outputs checked on the rows around the shard boundaries."""
        synth = self.synth
        jobs, full = {}, {}
        for name, (qt, w, x, y, rows) in self.cpu_jobs.items():
            if w is None:
                # Sharded configs: rank 0 regenerates the full matrix.
                key = "cfg1" if name == "cfg1" else "cfg4"
                if key not in full:
                    full[key] = (synth.kquant_blocks(qt, CFG["n"], CFG["k"], seed=CFG["seed_w"]) if key == "cfg1"
                                 else synth.kquant_blocks(qt, CFG4_N, CFG4_K, seed=1))
                w = full[key]
            jobs[name] = (qt, w, x, y, rows)
        return cpu_leg(jobs, time_it=self.world == 1)

    def report(self, cpu):
        h, world = self.head, self.world
        cpu_line = None
        if cpu is not None:
            res, topo = cpu
            for name, r in res.items():
                if name in self.configs:
                    self.configs[name]["err"] = r["err"]
                    self.configs[name]["err_elem"] = r["err_elem"]
            if "cfg1" in res:
                self.head_parity["max_rel_err_vs_oracle"] = res["cfg1"]["err"]
                self.head_parity["max_elem_rel_err_vs_oracle"] = res["cfg1"]["err_elem"]
            if world == 1 and "value" in res.get("cfg1", {}):
                c1 = res["cfg1"]
                cpu_line = {"value": c1["value"], "unit": c1["unit"], "cores": c1["cores"], "kind": "port",
                            "sample": f"{c1['calls']} full cfg1 GEMV calls ({c1['seconds']:.1f} s), C restatement of "
                                      f"the reference's AVX2 Q6K.Gemv, reference worker count {c1['cores']} "
                                      f"(CpuTopology.ChooseWorkerCount; {topo['logical']} logical CPUs)",
                            "configs": {n: {"v": r["value"], "u": r["unit"], "cores": r["cores"], "calls": r["calls"]}
                                        for n, r in res.items() if "value" in r and n != "cfg1"},
                            "host": topo}
        roofline = dict(h["roofline"])
        roofline["configs"] = self.configs
        for name, c in self.configs.items():
            parts = [f"# cfg {name}: {c['v']:.1f} {c['u']}"]
            if c.get("frac") is not None:
                parts.append(f"{c['frac']:.3f} of measured peak")
            if cpu_line and name in cpu_line["configs"]:
                cc = cpu_line["configs"][name]
                parts.append(f"cpu {cc['v']:.3g} {cc['u']} ({cc['cores']} cores)")
            if "err" in c:
                parts.append(f"err vs oracle {c['err']:.1e} (element-wise {c['err_elem']:.1e})")
            if "err_1gpu" in c:
                parts.append(f"err vs 1 GPU {c['err_1gpu']:.1e} bit-equal {c['bit_eq_1gpu']}, "
                             f"slices bit-equal to their rows alone {c['gather_exact']}")
            print(" | ".join(parts) + f" | {c['what']}")
        line = {
            "metric": METRIC, "value": h["value"], "unit": "GB/s", "n_gpus": world, "steps": self.args.steps,
            "warmup": self.args.warmup, "ms_per_step": h["ms_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": dict(CONFIG),
            "parallelism": (f"row-sharded N/{world} ({h['rows']} rows per GPU), gather {self.gather_desc} "
                            "(q35k_shard_matmul_dev)" if world > 1 else "single GPU"),
            "frac_of_nominal_8tbs": h["value"] / NOMINAL_HBM_GBS, "gemv_ms": h["gemv_ms"],
            "step_ms_events": h["step_ms"], "parity": self.head_parity, "roofline": roofline,
            "cpu_baseline": cpu_line, "e2e": h["e2e"], "clocks": h["clocks"],
            "gpu_launches": h["launches"] * self.args.steps, "launches_per_step": h["launches"],
        }
        line.update(h["extra"])
        print(json.dumps(line))

    def run(self):
        args = self.args
        self.headline()
        if self.world == 1 and not args.no_extra:
            self.gemv_configs()
            self.gemm_configs()
            self.argmax_config()
            self.ffn_config()
        if self.world > 1 and not args.no_extra:
            self.shard_configs()
        cpu = self.cpu_checks() if self.rank == 0 and not args.no_cpu else None
        if self.rank == 0:
            self.report(cpu)
        W, SW = self.head_w
        W.free()
        if self.world > 1:
            SW.free()
            self.group.close()
        self.ctx.close()
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


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
    "q6k_gemm_m512": (14, 512, 9728, 2560, 1.0, 0),
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
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU leg (baselines and oracle checks)")
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
        Bench(args).run()


if __name__ == "__main__":
    main()
