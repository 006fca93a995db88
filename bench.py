"""Benchmark of the MoE-layer hot path (H=2048, I=768, E=128, top-8, bf16).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl ours|reference]
                    [--ep-schedule c7|c6|c8] [--ep-transport peer|nccl] [--tp TP] [--zipf]

One step = one MoE-layer forward over T tokens.  At N=1 the workload is the
single-B200 fused MoE layer at T=16384 (router, sort, gather, w13+SwiGLU, w2,
combine) through ``moe_layer_forward``; ``value`` is tokens/s with inputs
resident in HBM, ``e2e`` the same through ``PermutedSparseMoE.forward`` with the
input copied from pinned host memory and the output copied back inside the
timed region.  At N>1 every rank runs an expert-parallel schedule with E/N
experts per rank: by default the all_to_all schedule (``EPSparseMoE``, C7
semantics) on its own T=16384 tokens (weak scaling); ``--ep-schedule c6`` the
replicated-input schedule with one all_reduce on T=4096 tokens, ``c8`` the
hybrid TP x EP schedule on T=16384 tokens (8 sequences x 2048) with
tp=``--tp`` (strong scaling, see ``ep_bench``).  ``--impl reference`` times
the reference algorithm's CPU restatement (the oracle) on the host cores on a
bounded sample of the same workload.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "MoE layer tokens/s (H=2048,I=768,E=128,top8,bf16), 1/2/4/8 B200, % of roofline"
H, I, E, K_TOP = 2048, 768, 128, 8
PEAKS_PATH = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return dict(FALLBACK_PEAKS), "fallback"


def layer_flops(T: int) -> float:
    return float(T) * (2 * H * E + K_TOP * 6 * H * I)


def layer_bytes(n_active: int, T: int) -> float:
    return n_active * 3 * H * I * 2 + 2 * H * E + 4 * T * H


# ----------------------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ----------------------------------------------------------------------------- inputs


def make_device_inputs(T: int, device, seed: int = 0, experts_per_rank: int = E, e0: int = 0):
    """Seeded synthetic inputs: x ~ N(0,1), weights ~ N(0, 0.02), bf16 on the device."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=device).to(bf)
    wr = (torch.randn(E, H, generator=g, device=device) * 0.02).to(bf)
    g2 = torch.Generator(device=device)
    g2.manual_seed(1000 + seed)
    wg = torch.empty(experts_per_rank, I, H, dtype=bf, device=device)
    wu = torch.empty_like(wg)
    wd = torch.empty(experts_per_rank, H, I, dtype=bf, device=device)
    for t in (wg, wu, wd):
        for e in range(experts_per_rank):
            t[e] = (torch.randn(t.shape[1:], generator=g2, device=device) * 0.02).to(bf)
    return x, wr, wg, wu, wd


# ----------------------------------------------------------------------------- CPU arm


def cpu_layer_sample(x, wr, wg, wu, wd, tokens: int, reps: int):
    """Time the torch restatement of PermutedSparseMoE.forward (C5) on the
    host cores: bf16 CPU tensors, every thread torch may use.  On the build
    container's CPU it runs at the speed of the unmodified reference C5 with
    an identical output (oracle/calibrate_port.py)."""
    from oracle.moe_torch_port import permuted_moe_torch
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    xs = x[:tokens]
    with torch.no_grad():
        permuted_moe_torch(xs, wr, wg, wu, wd, K_TOP)  # warm-up
        times = []
        for _ in range(reps):
            t0 = time.perf_counter()
            permuted_moe_torch(xs, wr, wg, wu, wd, K_TOP)
            times.append(time.perf_counter() - t0)
    return times, threads


def host_bf16(*ts):
    return [t.detach().to("cpu", torch.bfloat16).contiguous() for t in ts]


def run_reference(args):
    """--impl reference: the oracle port of the reference path on host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    T = args.tokens
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    x, wr, wg, wu, wd = make_device_inputs(min(T, 2048), dev)
    xb, wrb, wgb, wub, wdb = host_bf16(x, wr, wg, wu, wd)
    del x, wr, wg, wu, wd
    # Size each step's sample so that warm-up + steps stay within ~2 minutes.
    t_probe, threads = cpu_layer_sample(xb, wrb, wgb, wub, wdb, 64, 1)
    per_tok = t_probe[0] / 64
    budget = 100.0 / max(1, args.steps + args.warmup)
    tokens = int(max(8, min(2048, budget / max(per_tok, 1e-9))))
    times, threads = cpu_layer_sample(xb, wrb, wgb, wub, wdb, tokens, args.warmup + args.steps)
    times = times[args.warmup:] if len(times) > args.warmup else times
    total = sum(times)
    value = tokens * len(times) / total
    sample = (f"{tokens} of the {T} tokens per step (H=2048 I=768 E=128 k=8), torch bf16 "
              f"restatement of C5 PermutedSparseMoE.forward on the host cores, {len(times)} "
              "steps; it runs at the unmodified reference's speed on the build container's "
              "CPU (1.03x, identical output)")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": ("strong" if args.gpus > 1 and args.ep_schedule in ("c6", "c8", "c8block")
                    else "weak"),
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_block(T, args.gpus, args.ep_schedule, args.tp, args.zipf),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm


def config_block(T: int, n: int, schedule: str = "c7", tp: int = 1, zipf: bool = False) -> dict:
    per_rank = T
    if n == 1:
        wl = f"single-B200 fused MoE layer (C5/C9 path), T={T} tokens"
        par = "single"
    elif schedule == "c6":
        wl = (f"expert-parallel replicated-input MoE layer with one all_reduce (C6 path), "
              f"{T} tokens replicated on every rank, E/{n} experts per rank")
        par = f"ep{n} (replicated input)"
    elif schedule == "c8":
        per_rank = T // n
        wl = (f"hybrid TP x EP MoE layer (C8 path), {T} tokens in all, tp={tp} x dp={n // tp}, "
              f"a stripe of {per_rank} tokens per rank, E/{n} experts per rank, closing all_gather")
        par = f"tp{tp}xdp{n // tp}=ep{n}"
    elif schedule == "c8block":
        per_rank = T // n
        wl = (f"hybrid TP x EP decoder block (C8 HybridBlock: add+RMSNorm, TP GQA attention "
              f"32q/4kv heads of 128 over {T // 2048} sequences of 2048, add+RMSNorm, C8 MoE), "
              f"{T} tokens in all, tp={tp} x dp={n // tp}, E/{n} experts per rank")
        par = f"tp{tp}xdp{n // tp}=ep{n}"
    else:
        wl = f"expert-parallel all_to_all MoE layer (C7 path), {T} tokens per rank, E/{n} experts per rank"
        par = f"ep{n}"
    return {"workload": wl, "tokens_per_rank": per_rank, "hidden": H, "intermediate": I, "experts": E,
            "top_k": K_TOP,
            "routing": ("Zipf(1.2) skew: router N(0,0.02) + fp32 bias -1.2*ln(e+1)" if zipf
                        else "uniform (router N(0,0.02), no bias)"),
            "parallelism": par,
            "l2": "inputs larger than L2: 1.21 GB of expert weights streamed per step; "
                  "sweep: L2 flushed (512 MB write) before each timed replay"}


class Timer:
    def __init__(self, stream):
        self.stream = stream
        self.a = torch.cuda.Event(enable_timing=True)
        self.b = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        self.a.record(self.stream)
        return self

    def __exit__(self, *exc):
        self.b.record(self.stream)

    def ms(self):
        return self.a.elapsed_time(self.b)


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the gate/up GEMM at T=16384, taken from an ncu capture of that kernel on
# B200 (not measured by this script: CUDA events cannot count DRAM bytes).
# The weight bytes do not grow with T, so no other size is scaled from it.
W13_TRAFFIC = {(16384, 256): 1212910080 + 192624384}
W13_TRAFFIC_SOURCE = ("ncu capture of the same kernel at T=16384 "
                      "(dram__bytes_read.sum + dram__bytes_write.sum, one launch); "
                      "a recorded constant, not measured in this run")


def w13_kernel_name(tile_rows):
    if tile_rows == 256:
        return "grouped_gemm_pair_kernel<SwiGLU,6,gather> (w13, 2-CTA cluster)"
    return "grouped_gemm_kernel<BN,SwiGLU,stages,gather> (w13)"


SORT_CHUNK, SORT_THREADS, CLUSTER_SORT_MAX, CLUSTER_CHUNK = 2048, 256, 8, 4096
GEMV_W13_MAX_ROWS, ROUTER_SMALL_MAX_T = 128, 16
FUSED_DECODE_MAX_T, FUSED_DECODE_MAX_RECS = 16, 64


def sort_launches(R: int, e_local: int = E) -> int:
    """Kernels launch_sort_align issues for R records: one (single-CTA sort up
    to one 2048-record chunk, or one cluster of <= 8 CTAs of <= 4096 records
    each, i.e. R <= 32768) or three (histogram, scan, scatter)."""
    if R <= SORT_CHUNK and e_local <= SORT_THREADS:
        return 1
    chunk = -(-R // CLUSTER_SORT_MAX)
    chunk = -(-chunk // SORT_THREADS) * SORT_THREADS
    return 1 if chunk <= CLUSTER_CHUNK and e_local <= SORT_THREADS else 3


def layer_launches(T, tile_rows=None):
    """Kernels moe_layer_forward launches for T tokens.  Up to 64 records
    (T <= 8 at top-8): the single-launch decode layer.  Decode (T*k <= 128 records):
    router and sort fused in one kernel for T <= 16, the gate/up
    weight-streaming kernel, the down GEMV or GEMM, the combine.  Otherwise:
    router, sort (``sort_launches``), gate/up GEMM with the row gather fused,
    down GEMM, combine."""
    R = T * K_TOP
    if 0 < T <= FUSED_DECODE_MAX_T and R <= FUSED_DECODE_MAX_RECS:
        return 1
    if 0 < R <= GEMV_W13_MAX_ROWS:
        return (1 if T <= ROUTER_SMALL_MAX_T else 1 + sort_launches(R)) + 3
    return 1 + sort_launches(R) + 3


def e2e_pipelined(mod, x_host, dev, n_steps):
    """Milliseconds for n_steps layer calls through the public module, each
    step copying its input from pinned host memory and its result back to
    pinned host memory.  The copies run on two copy streams so that one
    step's input upload and the previous step's download overlap the current
    step's compute (double-buffered device inputs and host outputs); the
    events bracket the first upload and the last download."""
    compute = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    xd = [torch.empty(x_host.shape, dtype=x_host.dtype, device=dev) for _ in range(2)]
    y_host = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def run(n):
        for e in in_free + out_done:
            e.record(compute)
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(up):
                up.wait_event(in_free[b])
                xd[b].copy_(x_host, non_blocking=True)
                in_ready[b].record(up)
            compute.wait_event(in_ready[b])
            y = mod(xd[b])
            in_free[b].record(compute)
            out_ready[b].record(compute)
            with torch.cuda.stream(down):
                down.wait_event(out_ready[b])
                down.wait_event(out_done[b])
                y_host[b].copy_(y, non_blocking=True)
                y.record_stream(down)
                out_done[b].record(down)
        for e in out_done:
            compute.wait_event(e)

    run(2)
    torch.cuda.synchronize(dev)
    a = torch.cuda.Event(enable_timing=True)
    z = torch.cuda.Event(enable_timing=True)
    a.record(compute)
    run(n_steps)
    z.record(compute)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(z)


def run_ours_single(args):
    from moe_inference_verify_microbench_b200 import PermutedSparseMoE, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T = args.tokens
    peaks, peak_kind = load_peaks()
    x, wr, wg, wu, wd = make_device_inputs(T, dev)
    stream = torch.cuda.current_stream(dev)
    ws = torch.empty(ops.layer_workspace_bytes(T, H, I, E, K_TOP), dtype=torch.uint8, device=dev)
    y = torch.empty_like(x)

    def step():
        ops.moe_layer(x, wr, wg, wu, wd, K_TOP, out=y, workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_status(dev)

    clocks = ClockSampler(dev.index)
    clocks.start()
    time.sleep(0.3)
    # --- main timed region: whole layer through moe_layer_forward
    torch.cuda.synchronize()
    with Timer(stream) as tm:
        for _ in range(args.steps):
            step()
    torch.cuda.synchronize()
    ms_total = tm.ms()

    # --- per-kernel breakdown: the launches of moe_layer_forward, issued one C-ABI
    # call at a time into preallocated buffers, CUDA events between them.
    ev, n_active, tile_rows = kernel_breakdown(dev, x, wr, wg, wu, wd, T,
                                               max(3, min(args.steps, 50)))
    avg = {n: statistics.mean(v) for n, v in ev.items()}

    # --- e2e: PermutedSparseMoE.forward with host copies inside the timed region
    with torch.device(dev):
        mod = PermutedSparseMoE(H, I, E, K_TOP).to(torch.bfloat16)
    bwg, bwu, bwd = mod.pack()
    with torch.no_grad():
        mod.gate.weight.copy_(wr)
        bwg.copy_(wg)
        bwu.copy_(wu)
        bwd.copy_(wd)
    del wg, wu, wd
    x_host = x.cpu().pin_memory()
    n_e2e = max(3, min(args.steps, 100))
    with torch.no_grad():
        ms_e2e = e2e_pipelined(mod, x_host, dev, n_e2e)
    clk = clocks.stop()
    ops.check_status(dev)

    ms_step = ms_total / args.steps
    value = T / (ms_step * 1e-3)
    w13_flop = 2.0 * T * K_TOP * (2 * I) * H
    w13_tflops = w13_flop / (avg["w13"] * 1e-3) / 1e12
    peak_tc = peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"]
    t_roof = max(layer_flops(T) / (peak_tc * 1e12), layer_bytes(n_active, T) / (peaks["hbm_gbs"] * 1e9))
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded x~N(0,1), weights~N(0,0.02), random-init Qwen3-30B-A3B MoE shapes)",
        "config": config_block(T, 1),
        "roofline": {"bound": "tensor", "kernel": w13_kernel_name(tile_rows),
                     "achieved": w13_tflops, "peak": peak_tc, "unit": "TFLOP/s",
                     "frac": w13_tflops / peak_tc, "traffic": W13_TRAFFIC.get((T, tile_rows)),
                     "traffic_source": (W13_TRAFFIC_SOURCE if (T, tile_rows) in W13_TRAFFIC
                                        else "no ncu capture at this size"),
                     "peak_source": f"{peak_kind} bf16_tflops_sustained",
                     "algorithmic_per_launch": f"2*T*k*(2I)*H = {w13_flop:.4g} FLOP"},
        "layer_roofline": {"t_roof_ms": t_roof * 1e3, "frac": t_roof * 1e3 / ms_step,
                           "flop_per_step": layer_flops(T), "bytes_per_step": layer_bytes(n_active, T),
                           "active_experts": n_active},
        "breakdown_ms": {n: round(v, 5) for n, v in avg.items()},
        "e2e": {"value": T * n_e2e / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2,
                "api": "PermutedSparseMoE.forward", "steps": n_e2e,
                "pipelining": "step i+1's host->device copy and step i-1's device->host copy "
                              "run on their own streams (copy engines) while step i computes"},
        "gpu_launches": layer_launches(T, tile_rows) * args.steps,
        "clocks": clk,
    }
    if args.cpu_baseline:
        xb, wrb, wgb, wub, wdb = host_bf16(x[:1024], wr, bwg, bwu, bwd)
        times, threads = cpu_layer_sample(xb, wrb, wgb, wub, wdb, 1024, 3)
        line["cpu_baseline"] = {"value": 1024 / statistics.median(times), "unit": "tokens/s",
                                "cores": threads, "kind": "port",
                                "sample": "T=1024 tokens of the same weights, torch bf16 "
                                          "restatement of C5 PermutedSparseMoE.forward (runs at "
                                          "the reference's own speed), median of 3 after 1 "
                                          "warm-up"}
    if args.sweep:
        line["sweep_tokens_per_s"] = sweep(dev, [int(t) for t in args.sweep.split(",")], wr,
                                           bwg, bwu, bwd, peaks)
    print(json.dumps(line), flush=True)


def kernel_breakdown(dev, x, wr, wg, wu, wd, T, n_steps):
    """Per-kernel device time of the layer's own launch sequence at this size
    (router, sort into the layer's tile height, gate/up GEMM with the row
    gather fused, down GEMM, combine) through the C ABI, buffers preallocated
    so the host enqueues fast; a sleep kernel first lets the host fill the
    queue, so the events bracket GPU work only.  Returns (times, active
    experts, tile height)."""
    import ctypes

    from moe_inference_verify_microbench_b200 import _native, ops
    lib = _native.load()
    P = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    R = T * K_TOP
    rows = lib.moe_layer_tile_rows(T, H, I, E, K_TOP)
    i32, bf = torch.int32, torch.bfloat16
    ids = torch.empty(T, K_TOP, dtype=i32, device=dev)
    w = torch.empty(T, K_TOP, dtype=torch.float32, device=dev)
    mt = lib.moe_max_tiles_rows(R, E, rows)
    wsb = lib.moe_sort_align_workspace_bytes(R, E)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    counts = torch.empty(E, dtype=i32, device=dev)
    offs = torch.empty(E + 1, dtype=i32, device=dev)
    perm = torch.empty(R, dtype=i32, device=dev)
    tiles = torch.empty(mt, 4, dtype=i32, device=dev)
    nt = torch.empty(1, dtype=i32, device=dev)
    h = torch.empty(R, I, dtype=bf, device=dev)
    sl = torch.empty(R, H, dtype=bf, device=dev)
    y = torch.empty(T, H, dtype=bf, device=dev)
    st = ops.status_word(dev)
    S = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    names = ["router", "sort", "w13", "w2", "combine"]
    calls = [
        lambda: lib.moe_router_topk(P(x), P(wr), None, T, H, E, K_TOP, 1, P(ids), P(w), None, P(st), S),
        lambda: lib.moe_sort_align_rows(P(ids), R, E, 0, E, P(ws), wsb, P(counts), P(offs), None,
                                        P(perm), None, P(tiles), mt, P(nt), rows, P(st), S),
        lambda: lib.moe_grouped_w13_swiglu_gather_rows(P(x), T, P(perm), K_TOP, R, P(tiles), P(nt),
                                                       mt, P(wg), P(wu), E, H, I, P(h), rows,
                                                       P(st), S),
        lambda: lib.moe_grouped_w2_rows(P(h), R, P(tiles), P(nt), mt, P(wd), E, H, I, P(perm), P(w),
                                        P(sl), R, rows, P(st), S),
        lambda: lib.moe_combine(P(sl), R, None, None, None, 0, E, T, K_TOP, H, P(y), P(st), S),
    ]

    def one(marks):
        marks.append(torch.cuda.Event(enable_timing=True))
        marks[-1].record()
        for c in calls:
            rc = c()
            if rc != 0:
                raise RuntimeError(_native.error_string(rc))
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()

    for _ in range(3):
        one([])
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e6) * n_steps)
    all_marks = []
    for _ in range(n_steps):
        m = []
        one(m)
        all_marks.append(m)
    torch.cuda.synchronize()
    ops.check_status(dev)
    ev = {n: [m[i].elapsed_time(m[i + 1]) for m in all_marks] for i, n in enumerate(names)}
    n_active = int((counts > 0).sum().item())
    return ev, n_active, rows


def sweep(dev, token_counts, wr, wg, wu, wd, peaks):
    """Decode / prefill sweep: CUDA-graph-captured layer, inputs resident.  A
    512 MB buffer is written before every replay (outside the timed events), so
    each layer call finds the weights in HBM, not in the 126 MB L2.  Batches
    of up to 4 tokens are also timed on the one-pass decode layer (key
    "<T>_one_pass"), which takes the down weights transposed as well (built
    once, before any timing)."""
    from moe_inference_verify_microbench_b200 import ops
    out = {}
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    wdt = ops.transpose_down_weights(wd) if any(0 < t <= 4 for t in token_counts) else None
    runs = [(T, None) for T in token_counts] + [(T, wdt) for T in token_counts if 0 < T <= 4]
    for T, w_down_t in runs:
        g = torch.Generator(device=dev)
        g.manual_seed(T)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        ws = torch.empty(ops.layer_workspace_bytes(T, H, I, E, K_TOP), dtype=torch.uint8, device=dev)
        if w_down_t is not None:
            ws = torch.empty(ops.decode_layer_workspace_bytes(T, H, E), dtype=torch.uint8,
                             device=dev)
        y = torch.empty_like(x)
        for _ in range(3):
            ops.moe_layer(x, wr, wg, wu, wd, K_TOP, out=y, workspace=ws, w_down_t=w_down_t)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ops.moe_layer(x, wr, wg, wu, wd, K_TOP, out=y, workspace=ws, w_down_t=w_down_t)
        n = 50 if T <= 1024 else 20
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        evs = []
        for _ in range(n):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            graph.replay()
            b.record(stream)
            evs.append((a, b))
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        ids, _, _ = ops.router_topk(x, wr, K_TOP)
        n_act = int(torch.bincount(ids.reshape(-1).long(), minlength=E).gt(0).sum())
        peak_tc = peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"]
        t_roof = max(layer_flops(T) / (peak_tc * 1e12), layer_bytes(n_act, T) / (peaks["hbm_gbs"] * 1e9))
        out[str(T) + ("_one_pass" if w_down_t is not None else "")] = {
                       "tokens_per_s": T / (ms * 1e-3), "us_per_layer": ms * 1e3,
                       "roofline_frac": t_roof * 1e3 / ms, "active_experts": n_act,
                       "hbm_gbs": layer_bytes(n_act, T) / (ms * 1e-3) / 1e9}
        del graph
    del flush, wdt
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per step: 16384 (N=1; per rank for c7; in all for c8), "
                         "4096 replicated for c6")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ep-transport", choices=["peer", "nccl"], default="peer",
                    help="N>1: peer-store exchange over NVLink, or NCCL all_to_alls")
    ap.add_argument("--ep-schedule", choices=["c7", "c6", "c8", "c8block"], default="c7",
                    help="N>1: all_to_all (c7), replicated + all_reduce (c6), hybrid TP x EP (c8), "
                         "the whole C8 decoder block with attention (c8block)")
    ap.add_argument("--tp", type=int, default=2, help="c8: tensor-parallel group size")
    ap.add_argument("--zipf", action="store_true",
                    help="N>1: Zipf(1.2) router bias (the skewed-routing C7 configuration)")
    ap.add_argument("--ep-overlap", dest="ep_overlap", type=int, nargs="?", const=2, default=0,
                    metavar="CHUNKS",
                    help="N>1, peer transport: CHUNKS (default 2) token chunks, each chunk's "
                         "exchange overlapping the other chunks' GEMMs")
    ap.add_argument("--exchange-sms", type=int, default=16,
                    help="--ep-overlap: SMs the GEMMs leave to the exchange kernels")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--sweep", default="1,16,128,1024,4096",
                    help="comma-separated token counts for the graph-captured sweep ('' = none)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    multi = int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.gpus > 1
    if args.tokens is None:
        args.tokens = 4096 if multi and args.ep_schedule == "c6" else 16384
    if multi and args.ep_schedule in ("c8", "c8block"):
        n = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
        if args.tp < 1 or n % args.tp != 0 or args.tokens % n != 0:
            ap.error(f"c8 needs tp dividing N={n} and tokens divisible by N")
        if args.ep_schedule == "c8block" and (args.tokens // (n // args.tp)) % 2048 != 0:
            ap.error("c8block needs whole 2048-token sequences per TP group")
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 or args.gpus > 1:
        from moe_inference_verify_microbench_b200.ep_bench import run_ep
        run_ep(args, METRIC, config_block, ClockSampler)
        return
    run_ours_single(args)


if __name__ == "__main__":
    main()
