#!/usr/bin/env python3
"""Benchmark of the tinyqwen quantised decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Prints ONE JSON line (rank 0).  Workloads (synthetic seeded data of the BASELINE
shapes; random weights of the named architecture, no checkpoint):

  decode-qwen3-4b       (default) BASELINE config 4: Qwen3-4B-shaped i4 g64 model, fp16
                        KV, context 4096 filled by the engine's own greedy decode.  A step
                        is one decode token; value = device-timed ms/token of K
                        generate() steps; e2e = tqb200_engine_step per token (host token
                        in, host token out).  With --gpus N under torchrun the engine runs
                        tensor-parallel over the N ranks.
  decode-qwen2.5-0.5b   BASELINE config 2 shape (i4, fp32 KV, context 32).
  decode-qwen3-0.6b-vq2 BASELINE config 3 full step (VQ2 + BiIP, fp32 KV, context 32).
  matvec-i4             BASELINE config 1: i4 g64 matvec 4864x896.  A step is one
                        CUDA-graph replay of 64 launches, one per distinct copy of W
                        (64 x 2.45 MB = 157 MB > the 126 MB L2, so every launch streams W
                        from HBM).

Timing: W warm-up steps, then K steps bracketed by a barrier and a device sync, CUDA
events on the launching stream, max over ranks.  nvidia-smi clocks are sampled during
the timed region.  The reference's own CPU code (oracle/_ref, compiled from the
reference sources) is timed on a bounded sample for ``cpu_baseline``;
``--impl reference`` times only that.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tiny-llm_b200"))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------ distributed plumbing
def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=None)
        pg = dist
    return world, rank, local, pg


def share_nccl_id(pg, rank: int) -> bytes:
    """Rank 0's NCCL unique id (the engine's own communicator), broadcast to every rank."""
    import torch
    from tqb200 import lib
    nid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        nid.copy_(torch.frombuffer(bytearray(lib.nccl_unique_id()), dtype=torch.uint8))
    pg.broadcast(nid, src=0)
    return bytes(nid.cpu().numpy().tobytes())


def barrier(pg):
    if pg is not None:
        pg.barrier()


def max_over_ranks(pg, v: float) -> float:
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline
def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def ref_matvec_rate(seconds: float, threads: int):
    """Time the reference's matvec_i4_ref (oracle/_ref, the reference's own code) on
    config 1, rows split across `threads` host threads.  Returns (GB/s, kind, sample)."""
    from oracle.oracle import Oracle, RefLib
    from tqb200 import synth
    w, x = synth.config1_matvec(0)
    M, K, G = 4864, 896, 64
    rb = w.shape[1]
    if RefLib.available():
        lib, kind = RefLib(), "reference"
        fn = lib._matvec_i4
    else:
        lib, kind = Oracle(), "port"
        lib.set_threads(1)
        fn = lib._matvec_i4
    bounds = np.linspace(0, M, threads + 1).astype(int)
    y = np.zeros(M, np.float32)

    def one_call():
        ts = []
        for a, b in zip(bounds[:-1], bounds[1:]):
            if b <= a:
                continue
            wa = np.ascontiguousarray(w[a:b])
            ya = np.zeros(b - a, np.float32)
            ts.append((wa, ya))
        th = [threading.Thread(target=fn, args=(wa, x, ya, ya.size, K, G)) for wa, ya in ts]
        t0 = time.perf_counter()
        for t in th:
            t.start()
        for t in th:
            t.join()
        return time.perf_counter() - t0

    one_call()
    calls, spent = 0, 0.0
    while spent < seconds:
        spent += one_call()
        calls += 1
    bytes_per = M * rb + K * 4 + M * 4
    gbs = bytes_per * calls / spent / 1e9
    return gbs, kind, f"{calls} calls of matvec_i4_ref on config 1 (4864x896 g64) in {spent:.1f} s"


# ------------------------------------------------------------------ workloads
def matvec_graph_rate(tq, weights, x, M, K, G, reps: int, warmup: int, pdl: bool = True):
    """Device time of one tqb200_dev_matvec_i4_pdl launch (tqb200_dev_matvec_i4 with
    pdl=False: fully serialised launches): a CUDA graph of one launch per
    weight copy in `weights` (device tensors; together larger than L2, so every launch
    streams its matrix from HBM), replayed `reps` times between CUDA events on the
    launching stream.  Returns (us per launch, algorithmic GB/s, launches timed)."""
    import torch
    from tqb200 import lib
    dev = torch.device("cuda")
    dx = torch.from_numpy(x).to(dev)
    dy = torch.empty(M, device=dev)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    entry = tq.tqb200_dev_matvec_i4_pdl if pdl else tq.tqb200_dev_matvec_i4

    def launch_all():
        for wi in weights:
            st = entry(wi.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, G, sp)
            if st:
                raise lib.TQB200Error(st, tq.tqb200_last_error().decode())

    with torch.cuda.stream(stream):
        launch_all()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch_all()
    torch.cuda.synchronize()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    n = reps * len(weights)
    per_s = e0.elapsed_time(e1) / 1e3 / n
    algo = weights[0].numel() + K * 4 + M * 4
    del graph
    return per_s * 1e6, algo / per_s / 1e9, n


def matvec_single_call_us(tq, weights, x, M, K, G, calls: int = 50) -> float:
    """Median CUDA-event time of one launch by itself (no graph; rotating weight copies,
    so each call streams a matrix that is not in L2)."""
    import torch
    dev = torch.device("cuda")
    dx = torch.from_numpy(x).to(dev)
    dy = torch.empty(M, device=dev)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    ts = []
    with torch.cuda.stream(stream):
        for i in range(calls + 3):
            wi = weights[i % len(weights)]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            assert tq.tqb200_dev_matvec_i4(wi.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, G, sp) == 0
            e1.record(stream)
            e1.synchronize()
            if i >= 3:
                ts.append(e0.elapsed_time(e1) * 1e3)
    return float(np.median(ts))


def matvec_extras(pk, warmup: int) -> dict:
    """The metric's first clause beside a decode line: BASELINE config 1 (4864x896 g64,
    64 distinct copies per graph, plus single-call latency) and an lm_head-shaped i4
    matvec (151936x2560 g64, 218.8 MB per copy, two copies alternating)."""
    import torch
    from tqb200 import lib, synth
    tq = lib.load()
    dev = torch.device("cuda")
    out = {}
    w, x = synth.config1_matvec(0)
    rng = np.random.default_rng(1)
    ws = [torch.from_numpy(w).to(dev)] + [
        torch.from_numpy(synth.random_i4(rng, 4864, 896, 64) if i < 4 else w).to(dev)
        for i in range(1, 64)]
    us, gbs, n = matvec_graph_rate(tq, ws, x, 4864, 896, 64, 20, max(3, warmup))
    us_s, gbs_s, _ = matvec_graph_rate(tq, ws, x, 4864, 896, 64, 20, max(3, warmup), pdl=False)
    out["matvec_config1"] = {
        "shape": "4864x896 g64", "GB_per_s": round(gbs, 1), "us_per_launch": round(us, 3),
        "frac_of_hbm": round(gbs / pk["hbm_gbs"], 4), "launches_timed": n,
        "serialised_GB_per_s": round(gbs_s, 1), "serialised_us_per_launch": round(us_s, 3),
        "single_call_us": round(matvec_single_call_us(tq, ws, x, 4864, 896, 64), 3),
        "how": "CUDA graph of 64 tqb200_dev_matvec_i4_pdl launches over 64 distinct copies "
               "of W (157 MB > L2; each launch may read its weights while the previous "
               "finishes), CUDA events around 20 replays; serialised_*: the same with "
               "tqb200_dev_matvec_i4; single_call_us = median event time of one launch by "
               "itself"}
    del ws
    M, K = 151936, 2560
    ws = [torch.from_numpy(synth.random_i4_fast(rng, M, K, 64)).to(dev) for _ in range(2)]
    xl = rng.normal(size=K).astype(np.float32)
    us, gbs, n = matvec_graph_rate(tq, ws, xl, M, K, 64, 10, max(3, warmup))
    out["matvec_lm_head"] = {
        "shape": "151936x2560 g64", "GB_per_s": round(gbs, 1), "us_per_launch": round(us, 2),
        "frac_of_hbm": round(gbs / pk["hbm_gbs"], 4), "launches_timed": n,
        "how": "CUDA graph of 2 launches over 2 distinct copies (218.8 MB each > L2), "
               "CUDA events around 10 replays"}
    del ws
    torch.cuda.empty_cache()
    return out


def config_extras(args, pk, pk_kind) -> dict:
    """BASELINE configs 2, 3 and 5 beside the config-4 decode line, each through its own
    workload's bench at a short run (20 decode steps after 5 warm-up, or 5 prompts after
    3; its main numbers only; the full lines come from --workload <name>)."""
    import argparse as _ap
    out = {}
    runs = (("config2_decode", "decode-qwen2.5-0.5b", bench_decode),
            ("config3_decode", "decode-qwen3-0.6b-vq2", bench_decode),
            ("config5_prefill", "prefill-qwen3-30b-a3b", bench_prefill))
    for key, workload, fn in runs:
        sub = _ap.Namespace(**vars(args))
        sub.workload, sub.extras, sub.ctx, sub.layers = workload, False, None, None
        sub.steps, sub.warmup = (5, 3) if fn is bench_prefill else (20, 5)
        try:
            r = fn(sub, 0, None, pk, pk_kind)
        except Exception as ex:  # the main line still prints; the failure is recorded
            out[key] = {"workload": workload, "error": f"{type(ex).__name__}: {ex}"[:300]}
            continue
        e = {"workload": workload, "metric": r["metric"], "value": r["value"],
             "unit": r["unit"], "steps": sub.steps, "warmup": sub.warmup,
             "e2e": r["e2e"]["value"], "roofline_frac": r["roofline"]["frac"],
             "roofline_kernel": r["roofline"]["kernel"], "clocks": r["clocks"]}
        if "context" in r["config"]:
            e["context"] = r["config"]["context"]
        if "decode_after_prefill_ms_per_token" in r["config"]:
            e["decode_after_prefill_ms_per_token"] = r["config"]["decode_after_prefill_ms_per_token"]
        out[key] = e
    return out


def bench_matvec(args, rank, pg, pk, pk_kind):
    import torch
    from tqb200 import lib, synth
    tq = lib.load()
    G = 64
    cfg1 = args.rows is None and args.cols is None
    M, K = (4864, 896) if cfg1 else (args.rows or 4864, args.cols or 896)
    NCOPY = args.copies or (64 if cfg1 else 2)
    rng = np.random.default_rng(1)
    if cfg1:
        w, x = synth.config1_matvec(0)
    else:
        w, x = synth.random_i4_fast(rng, M, K, G), rng.normal(size=K).astype(np.float32)
    algo_bytes = w.nbytes + x.nbytes + M * 4
    dev = torch.device("cuda")
    ws = [torch.from_numpy(w).to(dev)]
    for i in range(1, NCOPY):   # distinct copies (same distribution) so L2 never holds W
        ws.append(torch.from_numpy(synth.random_i4(rng, M, K, G) if (i < 4 and cfg1) else
                                   synth.random_i4_fast(rng, M, K, G) if not cfg1 else w).to(dev))
    dx = torch.from_numpy(x).to(dev)
    dy = torch.empty(M, device=dev)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def graph_ms(entry):
        """Device ms of one replay of a graph of NCOPY launches of `entry`, over args.steps
        replays (clocks sampled during the timed replays)."""
        def launch_all():
            for wi in ws:
                st = entry(wi.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, G, sp)
                if st:
                    raise lib.TQB200Error(st, tq.tqb200_last_error().decode())

        with torch.cuda.stream(stream):
            launch_all()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch_all()
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
        clocks.start()
        barrier(pg)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        barrier(pg)
        ms = e0.elapsed_time(e1)
        clk = clocks.stop()
        del graph
        return max_over_ranks(pg, ms) / args.steps, clk

    # each launch with programmatic dependent launch (its weight loads start while the
    # previous launch finishes, as in a decode step), and each fully serialised
    ms_step, clk = graph_ms(tq.tqb200_dev_matvec_i4_pdl)
    ms_plain, _ = graph_ms(tq.tqb200_dev_matvec_i4)
    per_launch_s = ms_step / 1e3 / NCOPY
    achieved = algo_bytes / per_launch_s / 1e9
    plain_gbs = algo_bytes / (ms_plain / 1e3 / NCOPY) / 1e9
    world = int(os.environ.get("WORLD_SIZE", "1"))
    value = achieved * world  # replicas: every rank streams its own copies

    # e2e: the reference-facing host-pointer call (H2D of W and x, D2H of y per call)
    e2e = None
    if rank == 0:
        tq.tqb200_set_resident_weights(0)
        y = np.zeros(M, np.float32)
        for _ in range(3):
            lib.matvec_i4(w, x, M, K, G)
        n = 50
        t0 = time.perf_counter()
        for _ in range(n):
            st = tq.tqb200_matvec_i4(w, x, y, M, K, G)
            assert st == 0
        dt = (time.perf_counter() - t0) / n
        e2e = {"value": algo_bytes / dt / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(w.nbytes + x.nbytes),
               "d2h_bytes_per_step": int(M * 4), "note": "one tqb200_matvec_i4 host-pointer call per step"}
    out = {
        "metric": ("i4 matvec HBM GB/s (BASELINE config 1, 4864x896 g64)" if cfg1 else
                   f"i4 matvec HBM GB/s ({M}x{K} g64)"),
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u4 weights, f32 activations",
        "data": "synthetic (seeded, BASELINE config 1 distributions)",
        "config": {"workload": "matvec-i4 (config 1)" if cfg1 else f"matvec-i4 ({M}x{K})",
                   "rows": M, "cols": K, "group_size": G,
                   "launches_per_step": NCOPY, "distinct_weight_copies": NCOPY,
                   "l2": f"inputs larger than L2 ({NCOPY} distinct W copies, "
                         f"{NCOPY * w.nbytes / 1e6:.0f} MB)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": None, "peak_source": pk_kind,
                     "kernel": "i4_mv_tma_kernel<64>",
                     "algorithmic_bytes_per_launch": int(algo_bytes),
                     "how": "a CUDA graph of one tqb200_dev_matvec_i4_pdl launch per distinct "
                            "weight copy (each launch may read its weights while the previous "
                            "finishes; x and y after it), CUDA events around the replays"},
        "serialised": {"value": round(plain_gbs * world, 2), "unit": "GB/s",
                       "how": "the same graph of tqb200_dev_matvec_i4 launches (no overlap)"},
        "clocks": clk,
        "gpu_launches": NCOPY * args.steps,
        "e2e": e2e,
    }
    return out


# ------------------------------------------------------------------ prefill matmul
MM_SHAPE = (4096, 2048, 512, 64)  # config 5 q_proj over a 512-token prefill: M, K, N, G
MM_COPIES = 32                    # distinct weight copies per step (151 MB > L2)


def ref_matmul_rate(seconds: float):
    """The reference's matmul_i4_ref (oracle/_ref) on a column sample of MM_SHAPE, 1 core."""
    from oracle.oracle import Oracle, RefLib
    from tqb200 import synth
    M, K, N, G = MM_SHAPE
    rng = np.random.default_rng(7)
    w = synth.random_i4_fast(rng, M, K, G)
    n = 2
    x = rng.normal(size=(n, K)).astype(np.float32)
    lib, kind = (RefLib(), "reference") if RefLib.available() else (Oracle(), "port")
    lib.matmul_i4(w, x, M, K, n, G)
    calls, spent = 0, 0.0
    while spent < seconds:
        t0 = time.perf_counter()
        lib.matmul_i4(w, x, M, K, n, G)
        spent += time.perf_counter() - t0
        calls += 1
    tflops = 2.0 * M * K * n * calls / spent / 1e12
    return tflops, kind, (f"{calls} calls of matmul_i4_ref on {M}x{K} g{G} with {n} columns "
                          f"(of the workload's {N}) in {spent:.1f} s, 1 thread")


def bench_matmul(args, rank, pg, pk, pk_kind):
    """Tensor-core matmul_i4 (MatmulI4Fn) on the config-5 prefill q_proj shape."""
    import torch
    from tqb200 import lib, synth
    tq = lib.load()
    M, K, N, G = MM_SHAPE
    dev = torch.device("cuda")
    rng = np.random.default_rng(3)
    w0 = synth.random_i4_fast(rng, M, K, G)
    ws = [torch.from_numpy(w0).to(dev)]
    for _ in range(1, MM_COPIES):
        ws.append(torch.from_numpy(synth.random_i4_fast(rng, M, K, G)).to(dev))
    x = rng.normal(size=(N, K)).astype(np.float32)
    dx = torch.from_numpy(x).to(dev)
    dy = torch.empty(N, M, device=dev)
    scr = torch.empty(tq.tqb200_matmul_i4_scratch_bytes(M, K, N, G), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream

    def step():
        for wi in ws:
            st = tq.tqb200_dev_matmul_i4(wi.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, N, G,
                                         scr.data_ptr(), sp)
            if st:
                raise lib.TQB200Error(st, tq.tqb200_last_error().decode())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    barrier(pg)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier(pg)
    ms = max_over_ranks(pg, e0.elapsed_time(e1))
    clk = clocks.stop()
    per_call_s = ms / 1e3 / (args.steps * MM_COPIES)
    flops = 2.0 * M * N * K
    achieved = flops / per_call_s / 1e12
    world = int(os.environ.get("WORLD_SIZE", "1"))
    e2e = None
    if rank == 0:
        tq.tqb200_set_resident_weights(0)
        lib.matmul_i4(w0, x, M, K, N, G)
        n = 5
        t0 = time.perf_counter()
        for _ in range(n):
            lib.matmul_i4(w0, x, M, K, N, G)
        dt = (time.perf_counter() - t0) / n
        e2e = {"value": round(flops / dt / 1e12, 3), "unit": "TFLOP/s",
               "h2d_bytes_per_step": int(w0.nbytes + x.nbytes), "d2h_bytes_per_step": int(M * N * 4),
               "note": "one tqb200_matmul_i4 host-pointer call per step"}
    peak = pk.get("bf16_tflops", 1590.0)
    return {
        "metric": "i4 matmul TFLOP/s (tensor cores; BASELINE config 5 prefill q_proj, 4096x2048 g64, 512 tokens)",
        "value": round(achieved * world, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "u4 weights (exact bf16 codes), bf16 hi/lo activations, f32 accumulation",
        "data": "synthetic (seeded random codes/scales/zeros, N(0,1) activations)",
        "config": {"workload": "matmul-i4", "M": M, "K": K, "N": N, "group_size": G,
                   "calls_per_step": MM_COPIES,
                   "l2": f"inputs larger than L2 ({MM_COPIES} distinct weight copies, "
                         f"{MM_COPIES * w0.nbytes / 1e6:.0f} MB)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": pk_kind, "kernel": "mm_i4_tc_kernel<64>",
                     "note": "algorithmic 2*M*N*K flops over the whole call (weight repack and "
                             "activation pre-pass included); the MMAs issue 2.25x these flops"},
        "clocks": clk,
        "gpu_launches": 3 * MM_COPIES * args.steps,
        "e2e": e2e,
    }


# ------------------------------------------------------------------ decode (config 4)
DECODE_CTX = 4096


def matvec_bytes_by_kind(spec) -> dict:
    """Algorithmic bytes per decode step of every matvec kind: weights + x + y once
    (VQ2: codebook + one index byte per 4 weights; lm_head is i4 in every model here)."""
    from tqb200.synth import i4_row_bytes
    H, I, G = spec.hidden, spec.inter, spec.group_size
    qd, kvd, L = spec.n_heads * spec.head_dim, spec.n_kv_heads * spec.head_dim, spec.n_layers
    vq2 = spec.weight_dtype == "vq2"

    def mv(rows, cols, i4=False):
        w = rows * i4_row_bytes(cols, G) if (i4 or not vq2) else 2048 + rows * cols // 4
        return w + cols * 4 + rows * 4

    out = {"qkv": L * (mv(qd, H) + 2 * mv(kvd, H) - 2 * H * 4),
           "o_proj": L * (mv(H, qd) + H * 4),               # + residual read
           "gate_up": L * (2 * mv(I, H) - H * 4),
           "down": L * (mv(H, I) + I * 4 + H * 4),           # + up read (SwiGLU) + residual
           "lm_head": mv(spec.vocab, H, i4=True)}
    if spec.n_experts:  # MoE: the router and the k chosen experts' matrices per layer
        k, mi, E = spec.experts_per_tok, spec.moe_inter, spec.n_experts
        out["router"] = L * (E * H * 4 + H * 4 + E * 4)
        out["gate_up"] = L * (2 * mv(mi, H) * k - (2 * k - 1) * H * 4)
        out["down"] = L * k * mv(H, mi)
    return out


def step_bytes(spec, ctx: int, kv_bytes: int) -> int:
    mv = sum(matvec_bytes_by_kind(spec).values())
    kv = 2 * spec.n_layers * spec.n_kv_heads * ctx * spec.head_dim * kv_bytes
    return mv + kv


# DRAM bytes (read + written) of one step's matvec launches, from an ncu capture of one
# whole step (dram__bytes_read.sum + dram__bytes_write.sum over the step's
# i4_mv_tma_kernel launches, context 64: the matvec traffic does not depend on the
# context).  Reported per step, like `achieved`.
MATVEC_TRAFFIC_PER_STEP = {"decode-qwen3-4b": 2280930000}

# decode workloads: BASELINE configs 2, 3 (full step) and 4
DECODE_WORKLOADS = {
    "decode-qwen3-4b": dict(
        cfg="BASELINE config 4: Qwen3-4B-shaped i4 g64, fp16 KV", preset="QWEN3_4B", kv16=True,
        ctx=DECODE_CTX, dtype="u4 weights, f32 activations, f16 KV"),
    "decode-qwen2.5-0.5b": dict(
        cfg="BASELINE config 2: Qwen2.5-0.5B-shaped i4 g64, fp32 KV", preset="QWEN25_05B",
        kv16=False, ctx=32, dtype="u4 weights, f32 activations, f32 KV"),
    "decode-qwen3-30b-a3b": dict(
        cfg="BASELINE config 5 decode: Qwen3-30B-A3B-shaped MoE, i4 g64 experts, top-8 of 128, "
            "fp32 KV", preset="QWEN3_30B_A3B", kv16=False, ctx=576,
        dtype="u4 weights, f32 activations, f32 KV"),
    "decode-qwen3-0.6b-vq2": dict(
        cfg="BASELINE config 3 step: Qwen3-0.6B-shaped VQ2 + BiIP on every projection, fp32 KV",
        preset="QWEN3_06B_VQ2", kv16=False, ctx=32,
        dtype="2-bit VQ2 weights (i4 embed/lm_head), f32 activations, f32 KV"),
}


def decode_spec(wl: dict, max_seq: int):
    from dataclasses import replace
    from tqb200 import model as M
    base = getattr(M, wl["preset"])
    # i4 weights as random codes/scales/zeros (config-1 distributions) instead of RTN of
    # N(0,0.02): same bytes and shapes, built in seconds
    kw = {"weights": "codes"} if base.weight_dtype == "i4" else {}
    if base.n_experts:  # one layer's worth of expert tensors on the host, repeated (every
        kw["expert_layers"] = 1  # layer still gets its own device copy)
    return replace(base, max_seq_len=max_seq, **kw)


def bench_decode(args, rank, pg, pk, pk_kind):
    import torch
    from tqb200 import lib
    from tqb200.model import SynthModel
    lib.load()
    W, K = args.warmup, args.steps
    wl = DECODE_WORKLOADS[args.workload]
    ctx = args.ctx if args.ctx is not None else wl["ctx"]
    max_seq = ctx + 2 * W + 2 * K + 32  # + the stamped (W + K), e2e (19) and profiled (1) steps
    spec = decode_spec(wl, max_seq)
    if args.layers:
        from dataclasses import replace as _replace
        spec = _replace(spec, n_layers=args.layers)
    t0 = time.time()
    sm = SynthModel(spec, seed=0)
    t_build = time.time() - t0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp = {}
    if world > 1:  # tensor parallel: every projection's output rows sharded over the ranks
        tp = {"tp_size": world, "tp_rank": rank, "nccl_id": share_nccl_id(pg, rank)}
    eng = lib.Engine(sm, max_seq_len=max_seq, kv_fp16=wl["kv16"], **tp)
    exchange_mode = "none"
    if world > 1:
        exchange_mode = "nccl"
        if args.exchange == "p2p" and spec.weight_dtype != "vq2":
            # the all-gathers fused into the producing kernels (peer stores over NVLink)
            from tqb200 import exchange
            exchange.open_exchange(eng, exchange.gather_over_pg(eng.exchange_handle(), pg))
            exchange_mode = "p2p"
    del sm.tensors  # host copy no longer needed
    # KV for the context: run the engine itself over positions 0..ctx-W-1 (greedy)
    rng = np.random.default_rng(1)
    first = int(rng.integers(0, spec.vocab))
    toks, _ = eng.generate(first, ctx - W)
    tok = toks[-1]
    toks, _ = eng.generate(tok, W)   # warm-up steps (also captures the graph)
    tok = toks[-1]
    torch.cuda.synchronize()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    barrier(pg)
    torch.cuda.synchronize()
    toks, dev_ms = eng.generate(tok, K)  # K steps at the context, device-timed
    torch.cuda.synchronize()
    barrier(pg)
    clk = clocks.stop()
    dev_ms = max_over_ranks(pg, dev_ms)
    ms_step = dev_ms / K
    # the next K steps again, with the in-graph timeline: every launch in its stamped
    # form records the global timer (CTA in, past its dependency wait, out), so the
    # per-kernel in-step times come from graph replays of the same step (the stamps cost
    # a few percent, so the timed value above is taken without them)
    eng.set_timeline(K)
    toks, _ = eng.generate(toks[-1], W)   # also captures the stamped graph
    barrier(pg)
    toks, tl_ms = eng.generate(toks[-1], K)
    tl_ms = max_over_ranks(pg, tl_ms) / K
    tl_steps, tl_span, tl = eng.timeline()
    eng.set_timeline(0)

    # e2e: the C-ABI step call with host token in / host token out, every step
    tok = toks[-1]
    eng_steps = []
    for _ in range(3):
        tok = eng.step(tok)
    n_e2e = min(K, 16)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        tok = eng.step(tok)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
    # serialized per-kernel times (one step launched kernel by kernel, CUDA events between
    # launches, no PDL overlap): a diagnostic only, not the in-step times
    _, prof = eng.profile_step(tok)
    mvb = matvec_bytes_by_kind(spec)
    mv_bytes = sum(mvb.values())
    # in-step time of each kind: the timed steps' timeline, max over ranks
    excl = {k: max_over_ranks(pg, v[0]) for k, v in tl.items()}
    mv_ms = sum(excl.get(k, 0.0) for k in mvb)
    achieved = mv_bytes / (mv_ms * 1e-3) / 1e9
    kvb = 2 if wl["kv16"] else 4
    total_bytes = step_bytes(spec, ctx, kvb)
    kv_bytes = 2 * spec.n_layers * spec.n_kv_heads * ctx * spec.head_dim * kvb
    attn_io = spec.n_layers * (3 * spec.n_heads * spec.head_dim + 2 * spec.n_kv_heads * spec.head_dim) * 4
    attn_ms = excl.get("attention", 0.0)
    step_achieved = total_bytes / (ms_step * 1e-3) / 1e9
    # embed, per layer qkv / attention (QK-norm, RoPE and KV append fused) / o_proj /
    # gate_up / down, lm_head (+argmax), the device-side token feed, and with tensor
    # parallelism the cross-rank argmax (NCCL's all-gather kernels are not counted; with
    # the peer exchange there are none)
    # MoE layers: qkv, attention, o_proj, router (+ top-k), gate/up, down, combine
    per_layer = 7 if spec.n_experts else 5
    launches = 2 + per_layer * spec.n_layers + 1 + (1 if world > 1 else 0)
    out = {
        "metric": f"decode ms/token, batch 1 ({wl['cfg']}, ctx {ctx})",
        "value": round(ms_step, 4), "unit": "ms/token", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_step, 4), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": wl["dtype"],
        "data": f"synthetic (seeded random weights of the named shape; KV filled by the engine's "
                f"own greedy decode over {ctx} positions)",
        "config": {"workload": args.workload, "layers": spec.n_layers,
                   "hidden": spec.hidden, "inter": spec.inter, "heads": spec.n_heads,
                   "kv_heads": spec.n_kv_heads, "head_dim": spec.head_dim, "vocab": spec.vocab,
                   "context": ctx, "global_batch": 1,
                   "l2": "inputs larger than L2 (%.2f GB read per step)" % (total_bytes / 1e9),
                   "parallelism": "single GPU" if world == 1 else f"tp{world}",
                   "exchange": exchange_mode,
                   "bytes_per_step": int(total_bytes),
                   "hbm_floor_ms": round(total_bytes / (pk["hbm_gbs"] * 1e9) * 1e3, 4),
                   "model_build_s": round(t_build, 1)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": MATVEC_TRAFFIC_PER_STEP.get(args.workload),
                     "peak_source": pk_kind,
                     "kernel": ("vq2_matvec_kernel" if spec.weight_dtype == "vq2" else "i4_mv_tma_kernel")
                               + " (all matvecs of a step)",
                     "algorithmic_bytes_per_step": int(mv_bytes),
                     "matvec_ms_per_step": round(mv_ms, 4),
                     "how": "achieved = algorithmic_bytes_per_step / matvec_ms_per_step; "
                            "matvec_ms_per_step = the matvec launches' in-step time (in-graph "
                            "global-timer stamps: each launch from its first CTA past the "
                            "dependency wait to the next launch's, summed per step, averaged "
                            "over K stamped steps timed right after the K unstamped ones, whose "
                            "step time is in timeline.ms_per_step)",
                     "step_vs_hbm_floor": round((total_bytes / (pk["hbm_gbs"] * 1e9) * 1e3) / ms_step, 4)},
        "rooflines": {
            "attention": {"bound": "hbm", "achieved": round((kv_bytes + attn_io) / (attn_ms * 1e-3) / 1e9, 1)
                          if attn_ms > 0 else None,
                          "frac": round((kv_bytes + attn_io) / (attn_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4)
                          if attn_ms > 0 else None,
                          "algorithmic_bytes_per_step": int(kv_bytes + attn_io),
                          "attention_ms_per_step": round(attn_ms, 4),
                          "kernel": "attn_tma_kernel (QK-norm, RoPE and KV append fused)"},
            "step": {"bound": "hbm", "achieved": round(step_achieved, 1),
                     "frac": round(step_achieved / pk["hbm_gbs"], 4),
                     "algorithmic_bytes_per_step": int(total_bytes),
                     "note": "every byte a step must read (weights, KV at the context, "
                             "activations) over ms_per_step"}},
        "timeline_ms_by_kind": {k: {"in_step_ms": round(v[0], 4), "from_launch_ms": round(v[1], 4),
                                    "launches": v[2]} for k, v in tl.items()},
        "timeline": {"steps": tl_steps, "ms_per_step": round(tl_ms, 4),
                     "stamped_span_ms": round(tl_span, 4),
                     "in_step_ms_sum": round(sum(v[0] for v in tl.values()), 4),
                     "note": "in_step_ms: a launch's first CTA past its dependency wait to the "
                             "next stamped launch's (the step's last: to its last CTA out), so "
                             "the launches do not overlap and the sum <= ms_per_step; the "
                             "unstamped embed and token-feed kernels (and NCCL's) count with "
                             "the launch before them; from_launch_ms: first CTA in to last CTA "
                             "out (overlaps the previous kernel under programmatic dependent "
                             "launch)"},
        "kernel_ms_serialized": {k: round(v, 4) for k, v in prof.items() if v > 0},
        "clocks": clk,
        "gpu_launches": launches * K,
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms/token", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 8,
                "note": "tqb200_engine_step per token: token+position H2D, next token+status D2H"},
    }
    eng.close()
    del eng
    if world == 1 and args.extras:
        out.update(matvec_extras(pk, W))
        if args.workload == "decode-qwen3-4b":
            out.update(config_extras(args, pk, pk_kind))
    return out


# ------------------------------------------------------------------ prefill (config 5)
PREFILL_TOKENS = 512
PREFILL_DECODE_STEPS = 64
MATMUL_KINDS = ("qkv", "o_proj", "gate_up", "down")


def prefill_flops(spec, n: int) -> dict:
    """Algorithmic FLOPs of one n-token prefill at position 0, by part: the matmuls
    (2*M*K per token and matrix; experts: k chosen per token), the router, causal
    attention (QK^T and PV over n(n+1)/2 (query, key) pairs per head) and the last
    token's lm_head."""
    H, hd = spec.hidden, spec.head_dim
    qd, kvd = spec.n_heads * hd, spec.n_kv_heads * hd
    proj = 2.0 * n * (qd * H + 2 * kvd * H + H * qd)
    if spec.n_experts:
        ffn = 2.0 * n * spec.experts_per_tok * 3 * spec.moe_inter * H
        router = 2.0 * n * spec.n_experts * H
    else:
        ffn, router = 2.0 * n * 3 * spec.inter * H, 0.0
    attn = 4.0 * spec.n_heads * hd * (n * (n + 1) / 2)
    L = spec.n_layers
    return {"matmul": L * (proj + ffn), "router": L * router, "attention": L * attn,
            "lm_head": 2.0 * spec.vocab * H}


def bench_prefill(args, rank, pg, pk, pk_kind):
    """a 512-token prompt through the engine's batched prefill (every
    projection and the grouped experts on the tensor-core matmul), then 64 decode steps."""
    import torch
    from tqb200 import lib
    from tqb200.model import SynthModel
    lib.load()
    W, K = args.warmup, args.steps
    n = PREFILL_TOKENS
    wl = DECODE_WORKLOADS["decode-qwen3-30b-a3b"]
    spec = decode_spec(wl, n + PREFILL_DECODE_STEPS + 8)
    if args.layers:
        from dataclasses import replace as _replace
        spec = _replace(spec, n_layers=args.layers)
    t0 = time.time()
    sm = SynthModel(spec, seed=0)
    t_build = time.time() - t0
    world = int(os.environ.get("WORLD_SIZE", "1"))
    tp = {}
    if world > 1:  # expert parallelism: experts sharded, attention whole on every rank
        tp = {"tp_size": world, "tp_rank": rank, "nccl_id": share_nccl_id(pg, rank)}
    eng = lib.Engine(sm, max_seq_len=spec.max_seq_len, kv_fp16=False, **tp)
    if world > 1 and args.exchange == "p2p":  # the decode steps' expert-slot exchange
        from tqb200 import exchange
        exchange.open_exchange(eng, exchange.gather_over_pg(eng.exchange_handle(), pg))
    del sm.tensors
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, spec.vocab, n).astype(np.int32)
    ptr = C.c_void_p()
    lib._check(lib.load().tqb200_engine_stream(eng.h, C.byref(ptr)))
    stream = torch.cuda.ExternalStream(ptr.value)
    for _ in range(W):  # the first one also writes the prefill's weight tensor maps
        eng.reset()
        eng.prefill(prompt)
    torch.cuda.synchronize()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    clocks.start()
    barrier(pg)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        eng.reset()
        nxt = eng.prefill(prompt)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(pg)
    clk = clocks.stop()
    ms = max_over_ranks(pg, e0.elapsed_time(e1)) / K
    # e2e: the same C-ABI call timed on the host (token ids H2D, next token + status D2H)
    t0 = time.perf_counter()
    for _ in range(K):
        eng.reset()
        eng.prefill(prompt)
    e2e_ms = (time.perf_counter() - t0) * 1e3 / K
    # the config's 64 decode steps after the prompt
    toks, dec_ms = eng.generate(nxt, PREFILL_DECODE_STEPS)
    # live per-kind times of one prefill launched kernel by kernel
    eng.reset()
    _, prof = eng.profile_prefill(prompt)
    fl = prefill_flops(spec, n)
    mm_ms = sum(prof[k] for k in MATMUL_KINDS)
    achieved = fl["matmul"] / (mm_ms * 1e-3) / 1e12
    total_fl = sum(fl.values())
    peak = pk.get("bf16_tflops", 1590.0)
    L = spec.n_layers
    # embed; per MoE layer rmsnorm, pack, qkv, rope+kv, attention, pack, o_proj, rmsnorm,
    # router, top-k, plan, pack, gate/up, pack (+SwiGLU), down, combine; lm_head
    launches = 1 + 16 * L + 1
    out = {
        "metric": "prefill ms per 512-token prompt, batch 1 (BASELINE config 5: Qwen3-30B-A3B-"
                  "shaped MoE, i4 g64 experts, top-8 of 128, fp32 KV)",
        "value": round(ms, 3), "unit": "ms/prompt", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "u4 weights (exact bf16 codes), bf16 hi/lo activations, f32 accumulation; "
                 "f32 attention and KV",
        "data": "synthetic (seeded random weights of the named shape, 512 uniform random prompt ids)",
        "config": {"workload": args.workload, "layers": L, "hidden": spec.hidden,
                   "experts": spec.n_experts, "top_k": spec.experts_per_tok,
                   "expert_inter": spec.moe_inter, "heads": spec.n_heads,
                   "kv_heads": spec.n_kv_heads, "head_dim": spec.head_dim, "vocab": spec.vocab,
                   "prompt_tokens": n, "global_batch": 1,
                   "l2": "inputs larger than L2 (%.1f GB of expert weights read per prompt)"
                         % (L * spec.n_experts * 3 * spec.moe_inter * spec.hidden * 0.5625 / 1e9),
                   "parallelism": ("single GPU" if world == 1 else
                                   f"ep{world}: experts sharded, attention whole on every rank; "
                                   "the prompt's expert rows summed over NCCL"),
                   "model_build_s": round(t_build, 1),
                   "prefill_tflop": round(total_fl / 1e12, 4),
                   "prefill_tflops_whole_step": round(total_fl / (ms * 1e-3) / 1e12, 2),
                   "decode_after_prefill_ms_per_token": round(dec_ms / PREFILL_DECODE_STEPS, 4)},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "peak_source": pk_kind,
                     "kernel": "mm_i4_tc_kernel<64> (every projection and expert GEMM of a prompt)",
                     "algorithmic_flops_per_step": fl["matmul"],
                     "matmul_ms_per_step": round(mm_ms, 3),
                     "note": "algorithmic 2*M*N*K flops of the matmul launches over their summed "
                             "CUDA-event times; the MMAs issue 2.5x these flops (bf16 hi + lo "
                             "halves of X and the zero-term K step)"},
        "kernel_ms_by_kind": {k: round(v, 4) for k, v in prof.items() if v > 0},
        "clocks": clk,
        "gpu_launches": launches * K,
        "e2e": {"value": round(e2e_ms, 3), "unit": "ms/prompt", "h2d_bytes_per_step": 4 * (n + 1),
                "d2h_bytes_per_step": 8,
                "note": "tqb200_engine_prefill per prompt: position + ids H2D, next token + status D2H"},
    }
    eng.close()
    return out


def ref_prefill_rate(threads_note: str = ""):
    """Reference CPU cost of a 512-token config-5 prompt: forward_prefill of an i4 MoE model
    runs forward_token per token (runtime/qwen_forward_prefill.cpp:91-104; the batched MoE
    path is GPTQ-only), so the cost is 512 decode steps at contexts 0..511, sampled as
    the decode cost at the mean context 256."""
    ms, kind, sample = ref_decode_rate("decode-qwen3-30b-a3b", PREFILL_TOKENS // 2, threads_note)
    return ms * PREFILL_TOKENS, kind, (f"{PREFILL_TOKENS} x the per-token forward_token cost at "
                                       f"the mean context {PREFILL_TOKENS // 2}: " + sample)


def ref_decode_rate(workload: str, ctx: int, threads_note: str = ""):
    """Reference CPU decode cost per token for a decode workload (oracle/_ref: the
    reference's own QwenModel::forward_token and attention_decode_ref), bounded sample:
    2- and 6-layer models of the workload's shape give the per-layer and head costs (the
    step is a sum over layers plus the head, so it extrapolates exactly in layers);
    attention at the workload's context is timed separately with attention_decode_ref
    (fp32 KV: the reference's fp16-KV attention is aarch64-only) and added per layer."""
    import tempfile
    from dataclasses import replace
    from oracle.oracle import Oracle, RefLib
    from tqb200.model import SynthModel
    wl = DECODE_WORKLOADS[workload]
    base = decode_spec(wl, 64)
    have_ref = RefLib.available()
    times = {}
    la, lb = (2, 3) if base.n_experts else (2, 6)
    with tempfile.TemporaryDirectory() as td:
        for nl in (la, lb):
            spec = replace(base, n_layers=nl)
            sm = SynthModel(spec, seed=0)
            if have_ref:
                ref = RefLib()
                path = os.path.join(td, f"m{nl}.tqwen")
                sm.write_tqwen(path)
                m = ref.open_model(path, 64, spec.vocab, False)
            else:
                orc = Oracle()
                orc.set_threads(1)
                m = orc.model(sm, 64, False)
            m.step(1)
            best = float("inf")
            for i in range(3):
                t0 = time.perf_counter()
                m.step(2 + i)
                best = min(best, time.perf_counter() - t0)
            times[nl] = best
            m.close()
            del sm
    t_layer = (times[lb] - times[la]) / (lb - la)
    t_head = times[la] - la * t_layer
    # attention over the 4096-position KV of one layer vs the 4-position one above
    lib = RefLib() if have_ref else Oracle()
    H, KVH, hd = base.n_heads, base.n_kv_heads, base.head_dim
    rng = np.random.default_rng(0)
    q = rng.normal(size=H * hd).astype(np.float32)
    kc = rng.normal(size=KVH * ctx * hd).astype(np.float32)
    vc = rng.normal(size=KVH * ctx * hd).astype(np.float32)
    t0 = time.perf_counter()
    lib.attention(q, kc, vc, ctx, ctx, H, KVH, hd, 0.088)
    t_attn = time.perf_counter() - t0
    total = t_head + base.n_layers * (t_layer + t_attn)
    kind = "reference" if have_ref else "port"
    sample = (f"forward_token of {la}- and {lb}-layer {base.name} models at context ~4 "
              f"(best of 3: {times[la]*1e3:.0f} / {times[lb]*1e3:.0f} ms per token) extrapolated to "
              f"{base.n_layers} layers, plus attention_decode_ref at context {ctx} "
              f"({t_attn*1e3:.1f} ms per layer); 1 thread (the reference's x86 kernels are "
              f"single-threaded){threads_note}")
    return total * 1e3, kind, sample


def bench_reference_arm(args, rank):
    """--impl reference: the reference's own CPU code on the host cores."""
    if rank != 0:
        return None
    threads = cpu_threads()
    if args.workload.startswith("decode"):
        wl = DECODE_WORKLOADS[args.workload]
        ctx = args.ctx if args.ctx is not None else wl["ctx"]
        per = []
        for _ in range(max(1, min(args.steps, 2))):
            ms, kind, sample = ref_decode_rate(args.workload, ctx)
            per.append(ms)
        ms = float(np.median(per))
        return {
            "impl": "reference",
            "metric": f"decode ms/token, batch 1 ({wl['cfg']}, ctx {ctx})",
            "value": round(ms, 2), "unit": "ms/token", "n_gpus": 0, "steps": len(per),
            "warmup": 0, "ms_per_step": round(ms, 2), "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "quantised weights, f32 activations (double accumulation), f32 KV",
            "data": "synthetic (seeded random weights of the named shape)",
            "config": {"workload": args.workload, "context": ctx},
            "cpu_baseline": {"value": round(ms, 2), "unit": "ms/token", "cores": 1, "kind": kind,
                             "sample": sample + f"; host has {threads} threads"},
            "e2e": {"value": round(ms, 2), "unit": "ms/token", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    if args.workload == "prefill-qwen3-30b-a3b":
        ms, kind, sample = ref_prefill_rate(f"; host has {threads} threads")
        return {
            "impl": "reference",
            "metric": "prefill ms per 512-token prompt, batch 1 (BASELINE config 5: Qwen3-30B-A3B-"
                      "shaped MoE, i4 g64 experts, top-8 of 128, fp32 KV)",
            "value": round(ms, 1), "unit": "ms/prompt", "n_gpus": 0, "steps": 1, "warmup": 0,
            "ms_per_step": round(ms, 1), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "quantised weights, f32 activations (double accumulation), f32 KV",
            "data": "synthetic (seeded random weights of the named shape)",
            "config": {"workload": args.workload, "prompt_tokens": PREFILL_TOKENS},
            "cpu_baseline": {"value": round(ms, 1), "unit": "ms/prompt", "cores": 1, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(ms, 1), "unit": "ms/prompt", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    if args.workload == "matmul-i4":
        tf, kind, sample = ref_matmul_rate(max(2.0, 0.5 * args.steps))
        M, K, N, G = MM_SHAPE
        return {
            "impl": "reference",
            "metric": "i4 matmul TFLOP/s (tensor cores; BASELINE config 5 prefill q_proj, 4096x2048 g64, 512 tokens)",
            "value": round(tf, 6), "unit": "TFLOP/s", "n_gpus": 0, "steps": 1, "warmup": 0,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u4 weights, f32 activations (double accumulation)",
            "data": "synthetic (seeded random codes/scales/zeros, N(0,1) activations)",
            "config": {"workload": "matmul-i4", "M": M, "K": K, "N": N, "group_size": G},
            "cpu_baseline": {"value": round(tf, 6), "unit": "TFLOP/s", "cores": 1, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(tf, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    gbs, kind, sample = ref_matvec_rate(max(2.0, 0.5 * args.steps), threads)
    return {
        "impl": "reference",
        "metric": "i4 matvec HBM GB/s (BASELINE config 1, 4864x896 g64)",
        "value": round(gbs, 4), "unit": "GB/s", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u4 weights, f32 activations (double accumulation)",
        "data": "synthetic (seeded, BASELINE config 1 distributions)",
        "config": {"workload": "matvec-i4 (config 1)", "rows": 4864, "cols": 896, "group_size": 64},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode-qwen3-4b",
                    choices=list(DECODE_WORKLOADS) + ["matvec-i4", "matmul-i4",
                                                      "prefill-qwen3-30b-a3b"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ctx", type=int, default=None,
                    help="decode context in KV positions (default: the workload's)")
    ap.add_argument("--layers", type=int, default=None,
                    help="decode workloads: fewer layers than the model (small profiling cases)")
    ap.add_argument("--rows", type=int, default=None, help="matvec-i4: rows (default config 1)")
    ap.add_argument("--cols", type=int, default=None, help="matvec-i4: columns (default config 1)")
    ap.add_argument("--copies", type=int, default=None,
                    help="matvec-i4: distinct weight copies per graph (default 64 for config 1, else 2)")
    ap.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p",
                    help="tensor-parallel decode: all-gathers fused into the producing kernels "
                         "over peer memory (p2p, i4 models) or NCCL all-gather launches")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="decode workloads: skip the config-1 and lm_head matvec keys")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world, rank, local, pg = (int(os.environ.get("WORLD_SIZE", "1")),
                              int(os.environ.get("RANK", "0")),
                              int(os.environ.get("LOCAL_RANK", "0")), None)
    if args.impl == "reference":
        out = bench_reference_arm(args, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    import torch
    torch.cuda.set_device(local)
    world, rank, local, pg = dist_init()
    pk, pk_kind = peaks()
    if args.workload == "matvec-i4":
        out = bench_matvec(args, rank, pg, pk, pk_kind)
    elif args.workload == "matmul-i4":
        out = bench_matmul(args, rank, pg, pk, pk_kind)
    elif args.workload == "prefill-qwen3-30b-a3b":
        out = bench_prefill(args, rank, pg, pk, pk_kind)
    else:
        out = bench_decode(args, rank, pg, pk, pk_kind)
    if rank == 0:
        threads = cpu_threads()
        if args.workload == "matvec-i4":
            gbs, kind, sample = ref_matvec_rate(max(0.5, args.cpu_seconds), 1)
            out["cpu_baseline"] = {"value": round(gbs, 4), "unit": "GB/s", "cores": 1,
                                   "kind": kind, "sample": sample + f" (host has {threads} threads)"}
        elif args.workload == "matmul-i4":
            tf, kind, sample = ref_matmul_rate(max(1.0, args.cpu_seconds))
            out["cpu_baseline"] = {"value": round(tf, 6), "unit": "TFLOP/s", "cores": 1,
                                   "kind": kind, "sample": sample + f" (host has {threads} threads)"}
        elif args.workload == "prefill-qwen3-30b-a3b":
            if args.cpu_seconds > 0:
                ms, kind, sample = ref_prefill_rate(f"; host has {threads} threads")
                out["cpu_baseline"] = {"value": round(ms, 1), "unit": "ms/prompt", "cores": 1,
                                       "kind": kind, "sample": sample}
        elif args.cpu_seconds > 0:
            ms, kind, sample = ref_decode_rate(args.workload, out["config"]["context"],
                                               f"; host has {threads} threads")
            out["cpu_baseline"] = {"value": round(ms, 2), "unit": "ms/token", "cores": 1,
                                   "kind": kind, "sample": sample}
        print(json.dumps(out), flush=True)
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
