"""Multi-GPU leg of ``bench.py``: the C7 expert-parallel schedule
(``EPSparseMoE`` pure, all_to_all dispatch/combine; the peer-store exchange
over NVLink by default, NCCL all_to_alls with ``--ep-transport nccl``) with T
tokens per rank and E/N experts per rank, one process per GPU (weak scaling).

Timing: W warm-up steps, then K steps bracketed by a barrier and a device
synchronise on both sides, CUDA events on each rank's stream, the maximum
over ranks.  ``value`` = N·T / that time.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
import time

import torch
import torch.distributed as dist

H, I, E, K_TOP = 2048, 768, 128, 8


def _build(rank: int, world: int, dev: torch.device, T: int, transport: str):
    from .ep_pure import EPSparseMoE

    with torch.device(dev):
        mod = EPSparseMoE(H, I, E, K_TOP, world, rank, group=None, transport=transport,
                          max_tokens_per_rank=T).to(torch.bfloat16)
    wg, wu, wd = mod.pack()
    g = torch.Generator(device=dev)
    with torch.no_grad():
        g.manual_seed(0)  # replicated router
        mod.gate.weight.copy_((torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        for t in (wg, wu, wd):
            for e in range(t.shape[0]):
                g.manual_seed(1000 + 3 * (mod.expert_start + e) + (0 if t is wg else 1 if t is wu else 2))
                t[e].copy_((torch.randn(t.shape[1:], generator=g, device=dev) * 0.02).to(torch.bfloat16))
        g.manual_seed(10 + rank)  # distinct tokens per rank
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    return mod, x


def run_ep(args, metric, config_block, clock_sampler_cls) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # NCCL prints its version on stdout while communicators come up; keep stdout
    # for the one JSON line by pointing file descriptor 1 at stderr meanwhile.
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        dist.barrier()
        torch.cuda.synchronize()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    try:
        _run(args, metric, config_block, clock_sampler_cls, rank, world, dev)
        dist.barrier()
    finally:
        # No collective here: after a failure on one rank the others end on the
        # process-group timeout instead of waiting in a barrier forever.
        dist.destroy_process_group()


def _timed(fn, steps, stream):
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([a.elapsed_time(b)], device=stream.device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def _run(args, metric, config_block, clock_sampler_cls, rank, world, dev) -> None:
    from . import ops

    T = args.tokens
    transport = getattr(args, "ep_transport", "nccl")
    mod, x = _build(rank, world, dev, T, transport)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            mod(x)
        torch.cuda.synchronize()
        ops.check_status(dev)
        clocks = clock_sampler_cls(dev.index) if rank == 0 else None
        if clocks is not None:
            clocks.start()
            time.sleep(0.3)
        ms = _timed(lambda: mod(x), args.steps, stream)
        # Serial copies: with two ranks on one host, overlapping every rank's
        # upload and download with compute measured slower (6.5M against 8.4M
        # tokens/s at N=2) than upload, forward, download in turn.
        x_host = x.cpu().pin_memory()
        y_host = torch.empty_like(x_host).pin_memory()
        n_e2e = max(3, min(args.steps, 50))

        def e2e_step():
            y_host.copy_(mod(x_host.to(dev, non_blocking=True)), non_blocking=True)

        e2e_step()
        ms_e2e = _timed(e2e_step, n_e2e, stream)
        clk = clocks.stop() if clocks is not None else None
        ops.check_status(dev)
    mod.close()
    ms_step = ms / args.steps
    if rank != 0:
        return
    flop_rank = T * (2 * H * E + K_TOP * 6 * H * I)
    peaks = {}
    try:
        with open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                               "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
        src = "measured"
    except OSError:
        peaks = {"bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0}
        src = "fallback"
    peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
    achieved = flop_rank / (ms_step * 1e-3) / 1e12
    line = {
        "metric": metric, "value": world * T / (ms_step * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded x~N(0,1) per rank, weights~N(0,0.02))",
        "config": {**config_block(T, world), "ep_transport": transport},
        "roofline": {"bound": "tensor",
                     "kernel": f"whole EP layer per rank (compute + {transport} exchange)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": f"{src} bf16_tflops_sustained"},
        "e2e": {"value": world * T * n_e2e / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2,
                "api": f"EPSparseMoE.forward (C7 schedule, transport={transport})",
                "steps": n_e2e, "copies": "pinned host, upload / forward / download in "
                                          "turn on the compute stream; max over ranks"},
        # our kernels per forward: router, ep_keys, plan sort, local sort (3),
        # w13, w2, combine + (nccl) ep_meta, gather, partial combine
        #                   + (peer) publish, dispatch, recv wait, return, return wait
        "gpu_launches": (14 if transport == "peer" else 12) * args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
