"""Expert-parallel schedules (C6 lean all_reduce, C7 all_to_all, C8 hybrid)
on gloo CPU ranks, with a torch-CPU stand-in for the kernels, against the
reference's own outputs for the same inputs (tests/golden/ep_*.npz)."""

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, name, transport, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    from cpu_contract import CpuContractKernels, CpuPeerExchange
    from helpers import load_golden, to_t
    from moe_inference_verify_microbench_b200.ep_lean import EPSparseMoE as Lean
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from moe_inference_verify_microbench_b200.hybrid import HybridMoE
    from oracle import moe_oracle as mo

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = load_golden(name)
        T, H, I, E, k, tp = (int(g[n]) for n in ("T", "H", "I", "E", "k", "tp"))
        d = mo.make_inputs(T * world, H, I, E, int(g["seed"]))
        xall = to_t(d["x"])
        wr = to_t(d["wr"])
        wg = [to_t(d["w_gate"][e]) for e in range(E)]
        wu = [to_t(d["w_up"][e]) for e in range(E)]
        wd = [to_t(d["w_down"][e]) for e in range(E)]
        kind = str(g["kind"])
        overlap = int(transport[12:] or 2) if transport.startswith("peer_overlap") else 0
        tr = "peer" if overlap else transport
        if kind == "c6":
            mod = Lean(H, I, E, k, world, rank, group=None)
            x = xall[:T]
        elif kind == "c7":
            mod = Pure(H, I, E, k, world, rank, group=None, transport=tr, overlap=overlap)
            x = xall[rank * T:(rank + 1) * T]
        else:
            groups = [dist.new_group(list(range(i * tp, (i + 1) * tp))) for i in range(world // tp)]
            mod = HybridMoE(H, I, E, k, tp, rank % tp, groups[rank // tp], world, rank, None,
                            transport=tr, overlap=overlap)
            x = xall[(rank // tp) * T:(rank // tp + 1) * T]
        mod = mod.to(torch.bfloat16)
        mod._kernels = CpuContractKernels
        if transport == "peer":  # the exchange's buffer semantics, moved by gloo
            mod._peer = CpuPeerExchange(None, world * x.shape[0], H, k)
        if overlap:  # one exchange per token chunk, in program order on CPU
            from moe_inference_verify_microbench_b200.ep import _Streams
            part = -(-x.shape[0] // overlap)
            mod._peer_chunks = [CpuPeerExchange(None, world * part, H, k) for _ in range(overlap)]
            mod._streams = _Streams(torch.device("cpu"))
        mod.weight_loader(wr, wg, wu, wd)
        if int(g["zipf"]):
            lin = torch.nn.Linear(H, E, bias=True).to(torch.bfloat16)
            lin.weight.data.copy_(wr)
            lin.bias.data.copy_(torch.from_numpy(mo.zipf_bias(E)).to(torch.bfloat16))
            mod.gate = lin
        with torch.no_grad():
            y = mod(x)
            _, _, lg = CpuContractKernels.router_topk(x, mod.gate.weight, k, bias=getattr(mod.gate, "bias", None))
        srt = torch.sort(lg.float(), dim=-1, descending=True).values
        tie = (srt[:, k - 1] == srt[:, k]).numpy()
        yref = mo.f32_from_bf16_bits(g[f"y_rank{rank}"])
        err = mo.rel_err(y.float().numpy()[~tie], yref[~tie])
        q.put((rank, err, float(tie.mean())))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("name,world,transport", [
    ("ep_c6_w2.npz", 2, "nccl"), ("ep_c6_w4.npz", 4, "nccl"), ("ep_c7_w2.npz", 2, "nccl"),
    ("ep_c7_w4_zipf.npz", 4, "nccl"), ("ep_c8_w4_tp2.npz", 4, "nccl"),
    ("ep_c7_w2.npz", 2, "peer"), ("ep_c7_w4_zipf.npz", 4, "peer"),
    ("ep_c8_w4_tp2.npz", 4, "peer"),
    # eight ranks: C6 ep=8, C7 dp=ep=8 with the Zipf skew, C8 tp=4 x dp=2 and tp=2 x dp=4
    ("ep_c6_w8.npz", 8, "nccl"), ("ep_c7_w8_zipf.npz", 8, "nccl"),
    ("ep_c7_w8_zipf.npz", 8, "peer"), ("ep_c8_w8_tp4.npz", 8, "nccl"),
    ("ep_c8_w8_tp4.npz", 8, "peer"), ("ep_c8_w8_tp2.npz", 8, "peer"),
    # two token chunks, each exchange overlapping the other chunk's GEMMs
    ("ep_c7_w4_zipf.npz", 4, "peer_overlap"), ("ep_c8_w4_tp2.npz", 4, "peer_overlap"),
    ("ep_c7_w8_zipf.npz", 8, "peer_overlap"), ("ep_c7_w4_zipf.npz", 4, "peer_overlap3")])
def test_ep_schedule_matches_reference(name, world, transport):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + abs(hash((name, transport))) % 400
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, transport, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, tie in res:
        assert tie <= 0.2, (rank, tie)
        assert err <= 2e-2, (rank, err)


def test_overlap_needs_the_peer_transport():
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE
    with pytest.raises(ValueError):
        EPSparseMoE(64, 32, 8, 2, 1, 0, group=None, transport="nccl", overlap=True)


def test_unknown_transport_is_refused():
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE
    with pytest.raises(ValueError):
        EPSparseMoE(64, 32, 8, 2, 1, 0, group=None, transport="shm")


def test_peer_exchange_rejects_bad_shapes_before_touching_the_gpu():
    import torch
    from moe_inference_verify_microbench_b200.peer import PeerExchange
    for hidden, k, cap in ((100, 8, 64), (2048, 9, 64), (2048, 8, -1)):
        with pytest.raises(ValueError):
            PeerExchange(None, cap, hidden, k, torch.device("cpu"))


def _overcap_worker(rank, world, port, q):
    """Rank 1 passes twice the tokens the peer exchange was sized for; rank 0
    a batch within it.  Rank 1 must raise after taking part in the step (so
    rank 0's result is complete and both ranks stay in step), and a second
    forward within the capacity must then be correct on both ranks."""
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    from cpu_contract import CpuContractKernels, CpuPeerExchange
    from helpers import load_golden, to_t
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from oracle import moe_oracle as mo

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = load_golden("ep_c7_w2.npz")
        T, H, I, E, k = (int(g[n]) for n in ("T", "H", "I", "E", "k"))
        d = mo.make_inputs(T * world, H, I, E, int(g["seed"]))
        xall = to_t(d["x"])
        mod = Pure(H, I, E, k, world, rank, group=None, transport="peer",
                   max_tokens_per_rank=T).to(torch.bfloat16)
        mod._kernels = CpuContractKernels
        mod._peer = CpuPeerExchange(None, world * T, H, k)
        mod.weight_loader(to_t(d["wr"]), [to_t(d["w_gate"][e]) for e in range(E)],
                          [to_t(d["w_up"][e]) for e in range(E)],
                          [to_t(d["w_down"][e]) for e in range(E)])
        x = xall[rank * T:(rank + 1) * T]
        yref = mo.f32_from_bf16_bits(g[f"y_rank{rank}"])
        _, _, lg = CpuContractKernels.router_topk(x, mod.gate.weight, k)
        srt = torch.sort(lg.float(), dim=-1, descending=True).values
        keep = ~(srt[:, k - 1] == srt[:, k]).numpy()
        out = {}
        with torch.no_grad():
            if rank == 1:
                try:
                    mod(torch.cat([x, x]))
                    out["raised"] = False
                except ValueError:
                    out["raised"] = True
            else:
                y = mod(x)
                out["err_first"] = mo.rel_err(y.float().numpy()[keep], yref[keep])
            y = mod(x)
            out["err_second"] = mo.rel_err(y.float().numpy()[keep], yref[keep])
        q.put((rank, out))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_peer_batch_over_capacity_keeps_ranks_in_step():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29950
    procs = [ctx.Process(target=_overcap_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[1]["raised"] is True
    assert res[0]["err_first"] <= 2e-2
    assert res[0]["err_second"] <= 2e-2 and res[1]["err_second"] <= 2e-2


@pytest.mark.parametrize("name,world", [("ep_c6_w8.npz", 8), ("ep_c7_w8_zipf.npz", 8),
                                        ("ep_c8_w8_tp4.npz", 8), ("ep_c8_w4_tp2.npz", 4)])
def test_loopback_harness_on_cpu(name, world):
    """The thread-per-rank collective stand-in that the one-GPU expert-parallel
    test uses (tests/loopback.py), driven here with the CPU stand-in kernels:
    it must reproduce the reference's own per-rank outputs."""
    sys.path.insert(0, HERE)
    from cpu_contract import CpuContractKernels
    from helpers import load_golden, to_t
    from loopback import LoopbackWorld
    from moe_inference_verify_microbench_b200.ep_lean import EPSparseMoE as Lean
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from moe_inference_verify_microbench_b200.hybrid import HybridMoE
    from oracle import moe_oracle as mo
    import torch.distributed as dist

    g = load_golden(name)
    T, H, I, E, k, tp = (int(g[n]) for n in ("T", "H", "I", "E", "k", "tp"))
    kind = str(g["kind"])
    d = mo.make_inputs(T * world, H, I, E, int(g["seed"]))
    xall, wr = to_t(d["x"]), to_t(d["wr"])
    wg, wu, wd = (to_t(d[n]) for n in ("w_gate", "w_up", "w_down"))
    lw = LoopbackWorld(world, torch.device("cpu"))

    def rank_fn(rank):
        if kind == "c6":
            mod, x = Lean(H, I, E, k, world, rank, group=None), xall[:T]
        elif kind == "c7":
            mod, x = Pure(H, I, E, k, world, rank, group=None), xall[rank * T:(rank + 1) * T]
        else:
            groups = [dist.new_group(list(range(i * tp, (i + 1) * tp))) for i in range(world // tp)]
            mod = HybridMoE(H, I, E, k, tp, rank % tp, groups[rank // tp], world, rank, None)
            x = xall[(rank // tp) * T:(rank // tp + 1) * T]
        mod = mod.to(torch.bfloat16)
        mod._kernels = CpuContractKernels
        mod.weight_loader(wr, wg, wu, wd)
        if int(g["zipf"]):
            lin = torch.nn.Linear(H, E, bias=True).to(torch.bfloat16)
            lin.weight.data.copy_(wr)
            lin.bias.data.copy_(torch.from_numpy(mo.zipf_bias(E)).to(torch.bfloat16))
            mod.gate = lin
        with torch.no_grad():
            y = mod(x)
        _, _, lg = CpuContractKernels.router_topk(x, mod.gate.weight, k,
                                                  bias=getattr(mod.gate, "bias", None))
        srt = torch.sort(lg.float(), dim=-1, descending=True).values
        return y, (srt[:, k - 1] == srt[:, k]).numpy()

    for rank, (y, tie) in enumerate(lw.run(rank_fn)):
        yref = mo.f32_from_bf16_bits(g[f"y_rank{rank}"])
        assert tie.mean() <= 0.2
        assert mo.rel_err(y.float().numpy()[~tie], yref[~tie]) <= 2e-2, (name, rank)


def _ragged_overlap_worker(rank, world, port, q):
    """Rank r holds 0, 3, 7 or 13 tokens (empty and single-token chunks with
    four chunks); the chunked exchange must give exactly the one-chunk
    exchange's output on every rank, over two forwards."""
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    from cpu_contract import CpuContractKernels, CpuPeerExchange
    from helpers import to_t
    from moe_inference_verify_microbench_b200.ep import _Streams
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from oracle import moe_oracle as mo

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, I, E, k, n_max = 64, 32, 8, 2, 13
        d = mo.make_inputs(n_max * world, H, I, E, seed=5)
        weights = (to_t(d["wr"]), [to_t(d["w_gate"][e]) for e in range(E)],
                   [to_t(d["w_up"][e]) for e in range(E)], [to_t(d["w_down"][e]) for e in range(E)])
        mods = {}
        for chunks in (0, 4):
            m = Pure(H, I, E, k, world, rank, group=None, transport="peer",
                     max_tokens_per_rank=n_max, overlap=chunks).to(torch.bfloat16)
            m._kernels = CpuContractKernels
            m.weight_loader(*weights)
            if chunks:
                part = -(-n_max // chunks)
                m._peer_chunks = [CpuPeerExchange(None, world * part, H, k) for _ in range(chunks)]
                m._streams = _Streams(torch.device("cpu"))
            else:
                m._peer = CpuPeerExchange(None, world * n_max, H, k)
            mods[chunks] = m
        n = [0, 3, 7, 13][rank]
        x_all = to_t(d["x"])
        same = []
        with torch.no_grad():
            for step in range(2):
                x = x_all[rank * n_max + step:rank * n_max + step + n]
                same.append(bool(torch.equal(mods[4](x), mods[0](x))))
        q.put((rank, same))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_chunked_exchange_ragged_batches_equal_one_chunk():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ragged_overlap_worker, args=(r, 4, 29977, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same in res.items():
        assert all(same), (rank, same)
