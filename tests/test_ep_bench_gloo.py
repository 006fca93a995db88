"""The multi-GPU bench's per-schedule set-up (``ep_bench._build``) on two gloo
CPU ranks at small shapes, with the torch-CPU stand-in for the kernels: which
ranks share their input (C6 everywhere, C8 within a TP group, C7 nowhere),
that a global expert gets the same weights in every schedule, and that the
three schedules' forwards agree on the tokens they share."""

import os
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
T_SMALL, H_SMALL, I_SMALL, E_SMALL = 64, 256, 128, 16


def _worker(rank, world, port, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    from cpu_contract import CpuContractKernels
    from moe_inference_verify_microbench_b200 import ep_bench as eb
    from oracle import moe_oracle as mo

    eb.H, eb.I, eb.E = H_SMALL, I_SMALL, E_SMALL
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = {}
        dev = torch.device("cpu")
        for sched in ("c6", "c7", "c8"):
            mod, x = eb._build(rank, world, dev, T_SMALL, "nccl", sched, tp=2)
            mod._kernels = CpuContractKernels
            with torch.no_grad():
                y = mod(x)
            wg, _, wd = mod.pack()
            out[sched] = (x.float().numpy(), y.float().numpy(), mod.expert_start,
                          wg[0].float().numpy(), wd[-1].float().numpy())
        xs = {s: out[s][0] for s in out}
        res = {
            "shapes": {s: xs[s].shape for s in xs},
            "x_c6_eq_c7": bool((xs["c6"] == xs["c7"]).all()),
            "x_c6_eq_c8": bool((xs["c6"] == xs["c8"]).all()),
            "w_same": all((out["c6"][i] == out[s][i]).all() for s in ("c7", "c8") for i in (3, 4)),
            "start": {s: out[s][2] for s in out},
            "err_c7": mo.rel_err(out["c7"][1], out["c6"][1]) if rank == 0 else 0.0,
            "err_c8": mo.rel_err(out["c8"][1], out["c6"][1]),
        }
        # The skewed-routing C7 configuration: the router carries the Zipf bias,
        # so the first rank's experts take most of the records.
        mz, xz = eb._build(rank, world, dev, T_SMALL, "nccl", "c7", zipf=True)
        bias = mz.gate.bias.float()
        res["zipf_bias_ok"] = bool(torch.allclose(
            bias, eb.zipf_router_bias(E_SMALL).to(torch.bfloat16).float()))
        ids, _, _ = CpuContractKernels.router_topk(xz, mz.gate.weight, 4, bias=mz.gate.bias)
        res["zipf_low_share"] = float((ids < E_SMALL // world).float().mean())
        gathered = [None] * world
        dist.all_gather_object(gathered, [xs["c6"], xs["c7"]])
        res["c6_replicated"] = bool((gathered[0][0] == gathered[1][0]).all())
        res["c7_distinct"] = bool((gathered[0][1] != gathered[1][1]).any())
        q.put((rank, res))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_bench_schedules_build_consistent_inputs_and_agree():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, 29471, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, r in res.items():
        # c6: all T tokens on every rank; c7: T own tokens; c8 (tp=2, dp=1): T/dp tokens
        assert r["shapes"] == {"c6": (T_SMALL, H_SMALL), "c7": (T_SMALL, H_SMALL),
                               "c8": (T_SMALL, H_SMALL)}, r["shapes"]
        assert r["x_c6_eq_c8"], rank          # one TP group of two: the same tokens
        assert r["x_c6_eq_c7"] == (rank == 0), rank
        assert r["w_same"], rank
        assert all(v == rank * E_SMALL // world for v in r["start"].values()), r["start"]
        assert r["c6_replicated"] and r["c7_distinct"], r
        assert r["err_c7"] <= 2e-2 and r["err_c8"] <= 2e-2, (rank, r["err_c7"], r["err_c8"])
        assert r["zipf_bias_ok"] and r["zipf_low_share"] > 0.7, r["zipf_low_share"]


@pytest.mark.parametrize("sched,tp,per_rank,par", [
    ("c7", 1, 16384, "ep4"), ("c6", 1, 4096, "ep4 (replicated input)"),
    ("c8", 2, 4096, "tp2xdp2=ep4")])
def test_bench_config_names_the_schedule(sched, tp, per_rank, par):
    sys.path.insert(0, os.path.dirname(HERE))
    import bench
    T = 4096 if sched == "c6" else 16384
    c = bench.config_block(T, 4, sched, tp)
    assert c["tokens_per_rank"] == per_rank and c["parallelism"] == par
    assert c["routing"].startswith("uniform")
    assert bench.config_block(2048, 8, "c7", 1, True)["routing"].startswith("Zipf(1.2)")
    assert sched.upper() in c["workload"]


def test_bench_block_schedule_config_and_work():
    """The decoder-block schedule (HybridBlock at 8 x 2048 tokens): its config
    names the block and its FLOP count adds the attention of a rank's share
    (projections on 1/tp of the heads, causal attention over 2048 tokens)."""
    sys.path.insert(0, os.path.dirname(HERE))
    import bench
    from moe_inference_verify_microbench_b200.ep_bench import schedule_work
    c = bench.config_block(16384, 8, "c8block", 4)
    assert "HybridBlock" in c["workload"] and c["parallelism"] == "tp4xdp2=ep8"
    f, t, kind = schedule_work("c8block", 16384, 8, 4)
    moe = 2048 * 76_021_760
    proj = 2 * 2048 * (32 + 8) * 128 + 2 * 32 * 128 * 2048
    attn = 2 * 2048 * 128 * 32
    assert t == 16384 and kind == "strong"
    assert f == 8192 * (proj + attn) / 4 + moe


def test_roofline_arithmetic_matches_the_per_token_figures():
    """The FLOP counts behind every bench line's roofline: 76,021,760 FLOP per
    token for the layer (2·H·E router + 8 × 6·H·I experts), bytes = 9,437,184
    per active expert + the router weights + x read and y written."""
    sys.path.insert(0, os.path.dirname(HERE))
    import bench
    from moe_inference_verify_microbench_b200.ep_bench import schedule_work
    assert bench.layer_flops(1) == 76_021_760
    assert bench.layer_flops(16384) == 16384 * 76_021_760
    assert bench.layer_bytes(128, 16384) == 128 * 9_437_184 + 524_288 + 4 * 16384 * 2048
    assert bench.layer_launches(16384, 256) == 7 and bench.layer_launches(64, 128) == 5
    assert [bench.layer_launches(t) for t in (1, 4, 8, 9, 16, 1024, 4096, 8192)] == [
        1, 1, 1, 4, 4, 5, 5, 7]
    assert schedule_work("c7", 16384, 4) == (16384 * 76_021_760, 4 * 16384, "weak")
    f6, t6, s6 = schedule_work("c6", 4096, 4)
    assert (t6, s6) == (4096, "strong")
    assert f6 == 4096 * 2 * 2048 * 128 + 4096 * 8 * 6 * 2048 * 768 / 4
    assert schedule_work("c8", 16384, 4) == (4096 * 76_021_760, 16384, "strong")
