"""Multi-GPU leg of ``bench.py``: one of the three expert-parallel schedules
on N GPUs, one process per GPU, E/N experts per rank.

* ``c7`` (default): ``EPSparseMoE`` pure (C7/python/solution.py:65-269),
  all_to_all dispatch/combine with T tokens per rank (weak scaling); the
  peer-store exchange over NVLink by default, NCCL all_to_alls with
  ``--ep-transport nccl``; ``--zipf`` adds the Zipf(1.2) router bias of the
  skewed configuration (2048 tokens per rank: ``--tokens 2048 --zipf``).
  ``value`` = N·T / step time.
* ``c6``: ``EPSparseMoE`` lean (C6/python/solution.py:57-182), the same T
  tokens replicated on every rank, local experts only, one NCCL all_reduce
  of [T, H] (strong scaling).  ``value`` = T / step time.
* ``c8``: ``HybridMoE`` (C8/python/solution.py:59-230) with tp × dp = N:
  every TP group holds T/dp tokens, each rank runs the C7 core on its 1/tp
  stripe (T/N tokens) and the TP group all_gathers the stripes (strong
  scaling).  ``value`` = T / step time.
* ``c8block``: ``HybridBlock`` (C8/python/solution.py:235-325), the whole
  pre-norm decoder block (fused residual add + RMSNorms, TP GQA attention
  over 2048-token sequences with Qwen3-30B-A3B's 32 query / 4 KV heads of
  128, then the C8 MoE) on T/2048 sequences, tp × dp = N, each TP group
  holding T/dp tokens (strong scaling).  ``value`` = T / step time.

Timing: W warm-up steps, then K steps bracketed by a barrier and a device
synchronise on both sides, CUDA events on each rank's stream, the maximum
over ranks.
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
# Attention of the decoder block (Qwen3-30B-A3B): 32 query and 4 KV heads of
# 128, over sequences of 2048 tokens.
ATTN_HEADS, ATTN_KV_HEADS, ATTN_HEAD_DIM, ATTN_SEQ = 32, 4, 128, 2048


def zipf_router_bias(num_experts: int, s: float = 1.2) -> torch.Tensor:
    """The skewed-routing workload's router bias b_e = -s * ln(e + 1) (fp32,
    added to the logits before their bf16 rounding): expert e is picked with
    Zipf(s)-like frequency, so the ranks owning the low expert ids receive
    most of the rows."""
    e = torch.arange(num_experts, dtype=torch.float64)
    return (-s * torch.log(e + 1.0)).to(torch.float32)


def _build(rank: int, world: int, dev: torch.device, T: int, transport: str,
           schedule: str = "c7", tp: int = 1, zipf: bool = False, overlap: int = 0,
           exchange_sms: int = 16):
    """The schedule's module with seeded weights (the same global expert e gets
    the same weights on every rank and in every schedule) and this rank's
    input: T own tokens (c7), the T replicated tokens (c6), or the T/dp tokens
    of its TP group (c8).  ``zipf``: the router carries the Zipf(1.2) bias;
    ``overlap``: chunk count of the exchange that overlaps the GEMMs (peer
    only; 0 = one chunk, no overlap)."""
    from .ep import EPSparseMoELean, EPSparseMoEPure, HybridMoE

    x_rows, x_seed = T, 10 + rank
    moe_options = dict(transport=transport, max_tokens_per_rank=T // world, overlap=overlap,
                       exchange_sms=exchange_sms)
    with torch.device(dev):
        if schedule == "c8block":
            from .hybrid import HybridBlock
            groups = [dist.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(world // tp)]
            blk = HybridBlock(H, I, ATTN_HEADS, ATTN_KV_HEADS, ATTN_HEAD_DIM, E, K_TOP, tp, rank % tp,
                              groups[rank // tp], world, rank, None, **moe_options)
            blk = blk.to(torch.bfloat16)
            g = torch.Generator(device=dev)
            g.manual_seed(7)  # attention weights, the same on every rank before sharding
            qd, kvd = ATTN_HEADS * ATTN_HEAD_DIM, ATTN_KV_HEADS * ATTN_HEAD_DIM
            rnd = lambda *shape: (torch.randn(*shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            wq, wk, wv, wo = rnd(qd, H), rnd(kvd, H), rnd(kvd, H), rnd(H, qd)
            with torch.no_grad():
                blk.attn.qkv_proj.weight_loader(wq, "q")
                blk.attn.qkv_proj.weight_loader(wk, "k")
                blk.attn.qkv_proj.weight_loader(wv, "v")
                blk.attn.o_proj.weight_loader(wo)
            mod = blk.moe  # the MoE weights below; the block is returned
            x_rows, x_seed = T // (world // tp), 10 + rank // tp
        elif schedule == "c6":
            mod = EPSparseMoELean(H, I, E, K_TOP, world, rank, group=None)
            x_seed = 10  # replicated input
        elif schedule == "c8":
            # Every rank creates every TP group, in the same order.
            groups = [dist.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(world // tp)]
            mod = HybridMoE(H, I, E, K_TOP, tp, rank % tp, groups[rank // tp], world, rank, None,
                            transport=transport, max_tokens_per_rank=T // world,
                            overlap=overlap, exchange_sms=exchange_sms)
            x_rows, x_seed = T // (world // tp), 10 + rank // tp  # replicated within TP
        else:
            mod = EPSparseMoEPure(H, I, E, K_TOP, world, rank, group=None, transport=transport,
                                  max_tokens_per_rank=T, overlap=overlap,
                                  exchange_sms=exchange_sms)
        mod = mod.to(torch.bfloat16)
    wg, wu, wd = mod.pack()
    g = torch.Generator(device=dev)
    with torch.no_grad():
        g.manual_seed(0)  # replicated router
        mod.gate.weight.copy_((torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
        for t in (wg, wu, wd):
            for e in range(t.shape[0]):
                g.manual_seed(1000 + 3 * (mod.expert_start + e) + (0 if t is wg else 1 if t is wu else 2))
                t[e].copy_((torch.randn(t.shape[1:], generator=g, device=dev) * 0.02).to(torch.bfloat16))
        g.manual_seed(x_seed)
        x = torch.randn(x_rows, H, generator=g, device=dev).to(torch.bfloat16)
        if zipf:
            lin = torch.nn.Linear(H, E, bias=True, device=dev, dtype=torch.bfloat16)
            lin.weight.copy_(mod.gate.weight)
            lin.bias.copy_(zipf_router_bias(E).to(torch.bfloat16))
            mod.gate = lin
    if schedule == "c8block":
        return blk, x.reshape(x_rows // ATTN_SEQ, ATTN_SEQ, H)
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
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


def schedule_work(schedule: str, T: int, world: int, tp: int = 1):
    """(expected FLOP per rank, tokens of the whole job, scaling kind) of one
    step.  c7: every rank routes and computes its own T tokens (a rank's
    experts receive T·k records on average); c6: every rank routes all T
    replicated tokens and computes 1/N of their records; c8: every rank routes
    and computes its stripe of T/N tokens."""
    per_token = 2 * H * E + K_TOP * 6 * H * I
    if schedule == "c8block":
        # + attention per token of a rank's stripe: q/k/v/o projections on
        # 1/tp of the heads and causal attention (half of the 4·S·d per head)
        tp = max(1, tp)
        proj = 2 * H * (ATTN_HEADS + 2 * ATTN_KV_HEADS) * ATTN_HEAD_DIM + 2 * ATTN_HEADS * ATTN_HEAD_DIM * H
        attn = 2 * ATTN_SEQ * ATTN_HEAD_DIM * ATTN_HEADS
        tokens_tp_group = T // (world // tp)
        return tokens_tp_group * (proj + attn) / tp + (T // world) * per_token, T, "strong"
    if schedule == "c6":
        return T * 2 * H * E + T * K_TOP * 6 * H * I / world, T, "strong"
    if schedule == "c8":
        return (T // world) * per_token, T, "strong"
    return T * per_token, world * T, "weak"


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
    schedule = getattr(args, "ep_schedule", "c7")
    tp = getattr(args, "tp", 1) if schedule in ("c8", "c8block") else 1
    zipf = bool(getattr(args, "zipf", False))
    overlap = int(getattr(args, "ep_overlap", 0) or 0)
    if transport != "peer" or schedule == "c6":
        overlap = 0
    exchange_sms = int(getattr(args, "exchange_sms", 16))
    mod, x = _build(rank, world, dev, T, transport, schedule, tp, zipf, overlap, exchange_sms)
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
    close = getattr(mod, "close", None)
    if close is not None:
        close()
    ms_step = ms / args.steps
    if rank != 0:
        return
    flop_rank, job_tokens, scaling = schedule_work(schedule, T, world, tp)
    if schedule == "c6":
        api = "EPSparseMoE.forward (C6 lean schedule, NCCL all_reduce)"
        exchange = "NCCL all_reduce"
        launches = 7  # router, sort (3), gate/up, down, masked combine
    elif schedule == "c8block":
        api = f"HybridBlock.forward (C8 block, tp={tp}, transport={transport})"
        exchange = f"{transport} exchange + NCCL all_gather + attention all_reduce"
        # two add_rmsnorm rows kernels + the C8 MoE's launches (below); the
        # attention's projections and SDPA are torch (cuBLAS / flash) kernels
        launches = 2 + (14 if transport == "peer" else 12) + (13 * (overlap - 1) if overlap else 0)
    else:
        api = (f"EPSparseMoE.forward (C7 schedule, transport={transport})" if schedule == "c7" else
               f"HybridMoE.forward (C8 schedule, tp={tp}, transport={transport})")
        exchange = f"{transport} exchange" + (" + NCCL all_gather" if schedule == "c8" else "")
        # router, ep_keys, plan sort, local sort (3), gate/up, down, combine
        # + (nccl) ep_meta, gather, partial combine
        # + (peer) publish, dispatch, recv wait, return, return wait
        # + (overlap) every further chunk's ep_keys, plan sort, local sort (3),
        #   gate/up, down, combine and exchange (5)
        launches = 14 if transport == "peer" else 12
        if overlap:
            launches += 13 * (overlap - 1)
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
    config = config_block(T, world, schedule, tp, zipf)
    if schedule != "c6":
        config["ep_transport"] = transport
        if overlap:
            config["ep_overlap"] = f"{overlap} token chunks, GEMMs on all but {exchange_sms} SMs"
    line = {
        "metric": metric, "value": job_tokens / (ms_step * 1e-3), "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded x~N(0,1), weights~N(0,0.02))",
        "config": config,
        "roofline": {"bound": "tensor",
                     "kernel": f"whole EP layer per rank (compute + {exchange})",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": f"{src} bf16_tflops_sustained",
                     "algorithmic_per_launch": f"expected FLOP per rank per step = {flop_rank:.4g}"},
        "e2e": {"value": job_tokens * n_e2e / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                "api": api, "steps": n_e2e,
                "copies": "pinned host, upload / forward / download in turn on the compute "
                          "stream; max over ranks; bytes per rank"},
        "gpu_launches": launches * args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
