"""Expert-parallel schedules on real GPUs over NCCL (one process per GPU):
C6 lean all_reduce, C7 all_to_all and C8 HybridMoE, against the reference's
own outputs (tests/golden/ep_*.npz) and, at the benchmark's shapes, against
the single-GPU layer.  Skipped when fewer GPUs than ranks are visible."""

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
pytestmark = pytest.mark.gpu


def _need(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    return dev


def _check_fixture(rank, world, dev, name, transport):
    """One rank's forward of the fixture's schedule on its transport: (relative
    error against the reference's own output on tokens without a top-k
    boundary tie, fraction of tied tokens)."""
    import torch.distributed as dist
    from helpers import load_golden, to_t
    from moe_inference_verify_microbench_b200 import ops
    from moe_inference_verify_microbench_b200.ep_lean import EPSparseMoE as Lean
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from moe_inference_verify_microbench_b200.hybrid import HybridMoE
    from oracle import moe_oracle as mo

    g = load_golden(name)
    T, H, I, E, k, tp = (int(g[n]) for n in ("T", "H", "I", "E", "k", "tp"))
    d = mo.make_inputs(T * world, H, I, E, int(g["seed"]))
    xall = to_t(d["x"], dev)
    wr = to_t(d["wr"], dev)
    wg = [to_t(d["w_gate"][e], dev) for e in range(E)]
    wu = [to_t(d["w_up"][e], dev) for e in range(E)]
    wd = [to_t(d["w_down"][e], dev) for e in range(E)]
    kind = str(g["kind"])
    overlap = int(transport[12:] or 2) if transport.startswith("peer_overlap") else 0
    tr = "peer" if overlap else transport
    with torch.device(dev):
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
    mod.weight_loader(wr, wg, wu, wd)
    bias = None
    if int(g["zipf"]):
        lin = torch.nn.Linear(H, E, bias=True).to(torch.bfloat16).to(dev)
        lin.weight.data.copy_(wr)
        lin.bias.data.copy_(torch.from_numpy(mo.zipf_bias(E)).to(torch.bfloat16))
        mod.gate = lin
        bias = lin.bias.float()
    with torch.no_grad():
        y = mod(x.contiguous())
        _, _, lg = ops.router_topk(x.contiguous(), mod.gate.weight, k, bias=bias, return_logits=True)
    torch.cuda.synchronize()
    ops.check_status(dev)
    srt = torch.sort(lg.float(), dim=-1, descending=True).values
    tie = (srt[:, k - 1] == srt[:, k]).cpu().numpy()
    yref = mo.f32_from_bf16_bits(g[f"y_rank{rank}"])
    if hasattr(mod, "close"):
        mod.close()
    dist.barrier()
    return mo.rel_err(y.float().cpu().numpy()[~tie], yref[~tie]), float(tie.mean())


def _fixture_worker(rank, world, port, name, transport, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    dev = _init(rank, world, port)
    try:
        err, tie = _check_fixture(rank, world, dev, name, transport)
        q.put((rank, err, tie))
    finally:
        dist.destroy_process_group()


def _spawn(target, world, args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("name,world,transport", [
    ("ep_c6_w2.npz", 2, "nccl"), ("ep_c7_w2.npz", 2, "nccl"), ("ep_c7_w2.npz", 2, "peer"),
    ("ep_c6_w4.npz", 4, "nccl"), ("ep_c7_w4_zipf.npz", 4, "nccl"),
    ("ep_c7_w4_zipf.npz", 4, "peer"), ("ep_c8_w4_tp2.npz", 4, "nccl"),
    ("ep_c8_w4_tp2.npz", 4, "peer"),
    ("ep_c6_w8.npz", 8, "nccl"), ("ep_c7_w8_zipf.npz", 8, "nccl"),
    ("ep_c7_w8_zipf.npz", 8, "peer"), ("ep_c8_w8_tp2.npz", 8, "nccl"),
    ("ep_c8_w8_tp2.npz", 8, "peer"), ("ep_c8_w8_tp4.npz", 8, "nccl"),
    ("ep_c8_w8_tp4.npz", 8, "peer")])
def test_ep_schedule_on_gpus_matches_reference(name, world, transport):
    _need(world)
    res = _spawn(_fixture_worker, world, (29800 + world + 10 * (transport == "peer"), name,
                                          transport))
    for rank, err, tie in res:
        assert tie <= 0.2, (rank, tie)
        assert err <= 2e-2, (rank, err)


def _full_worker(rank, world, port, kind, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    from moe_inference_verify_microbench_b200 import ops
    from moe_inference_verify_microbench_b200.ep_lean import EPSparseMoE as Lean
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from oracle import moe_oracle as mo

    dev = _init(rank, world, port)
    try:
        H, I, E, k, T = 2048, 768, 128, 8, 1024
        g = torch.Generator(device=dev)
        g.manual_seed(3)
        x_all = torch.randn(T * world, H, generator=g, device=dev).to(torch.bfloat16)
        wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wg = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wu = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        wd = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        with torch.device(dev):
            cls = Lean if kind == "c6" else Pure
            mod = cls(H, I, E, k, world, rank, group=None).to(torch.bfloat16)
        mod.weight_loader(wr, list(wg), list(wu), list(wd))
        x = x_all[:T] if kind == "c6" else x_all[rank * T:(rank + 1) * T]
        with torch.no_grad():
            y = mod(x.contiguous())
            y_single = ops.moe_layer(x.contiguous(), wr, wg, wu, wd, k)
        torch.cuda.synchronize()
        ops.check_status(dev)
        q.put((rank, mo.rel_err(y.float().cpu().numpy(), y_single.float().cpu().numpy())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["c6", "c7"])
def test_ep_full_shapes_match_single_gpu_layer(kind):
    _need(2)
    world = min(torch.cuda.device_count(), 8)
    res = _spawn(_full_worker, world, (29900 + (kind == "c7"), kind))
    for rank, err in res:
        assert err <= 1e-2, (rank, err)


def _check_peer_vs_nccl(rank, world, dev):
    """Four forwards with ragged per-rank token counts on both transports and
    on the peer transport with the two- and three-chunk overlapped exchange: whether
    each peer output is bit-identical to the NCCL one."""
    import torch.distributed as dist
    from moe_inference_verify_microbench_b200 import ops
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure

    H, I, E, k, T = 2048, 768, 128, 8, 2048
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wg = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wu = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    mods = {}
    for name, tr, ov in (("nccl", "nccl", 0), ("peer", "peer", 0), ("overlap", "peer", 2),
                         ("overlap3", "peer", 3)):
        with torch.device(dev):
            mods[name] = Pure(H, I, E, k, world, rank, group=None, transport=tr,
                              overlap=ov).to(torch.bfloat16)
        mods[name].weight_loader(wr, list(wg), list(wu), list(wd))
    same = []
    g.manual_seed(100 + rank)
    with torch.no_grad():
        for step in range(4):  # epochs; ragged token counts per step and rank
            n = T - 97 * ((step + rank) % 3)
            x = torch.randn(n, H, generator=g, device=dev).to(torch.bfloat16)
            dist.barrier()
            y_peer = mods["peer"](x)
            y_over = mods["overlap"](x)
            y_over3 = mods["overlap3"](x)
            y_nccl = mods["nccl"](x)
            same.append(bool(torch.equal(y_peer, y_nccl)))
            same.append(bool(torch.equal(y_over, y_nccl)))
            same.append(bool(torch.equal(y_over3, y_nccl)))
    torch.cuda.synchronize()
    ops.check_status(dev)
    for name in ("peer", "overlap", "overlap3"):
        mods[name].close()
    dist.barrier()
    return same


def _peer_worker(rank, world, port, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    dev = _init(rank, world, port)
    try:
        q.put((rank, _check_peer_vs_nccl(rank, world, dev)))
    finally:
        dist.destroy_process_group()


EP_FIXTURES = {2: ["ep_c6_w2.npz", "ep_c7_w2.npz"],
               4: ["ep_c6_w4.npz", "ep_c7_w4_zipf.npz", "ep_c8_w4_tp2.npz"],
               8: ["ep_c6_w8.npz", "ep_c7_w8_zipf.npz", "ep_c8_w8_tp2.npz", "ep_c8_w8_tp4.npz"]}


def _all_worker(rank, world, port, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    dev = _init(rank, world, port)
    try:
        res = {}
        for name in EP_FIXTURES[world]:
            for tr in (("nccl",) if "_c6_" in name else ("nccl", "peer", "peer_overlap")):
                res[f"{name}/{tr}"] = _check_fixture(rank, world, dev, name, tr)
        res["peer_bits_equal_nccl"] = _check_peer_vs_nccl(rank, world, dev)
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_all_schedules_in_one_process_group(world):
    """Every expert-parallel fixture of this world size (C6; C7 and C8 on both
    transports) against the reference's own per-rank outputs, and the peer
    transport bit-identical to NCCL, in ONE process group: the same checks
    as the per-fixture tests, for a fraction of their start-up cost."""
    _need(world)
    res = _spawn(_all_worker, world, (29700 + world,))
    for rank, r in res:
        for key, v in r.items():
            if key == "peer_bits_equal_nccl":
                assert all(v), (rank, v)
            else:
                err, tie = v
                assert tie <= 0.2, (rank, key, tie)
                assert err <= 2e-2, (rank, key, err)


@pytest.mark.parametrize("world", [2, 8])
def test_ep_peer_transport_bit_identical_to_nccl(world):
    """The peer-store exchange and the NCCL all_to_alls sum the same rows in
    the same order: outputs must be bit-identical, over several forwards
    with different per-rank token counts."""
    _need(world)
    res = _spawn(_peer_worker, world, (29950 + world,))  # both transports: same tile height
    for rank, same in res:
        assert all(same), (rank, same)


def _block_worker(rank, world, port, q):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    import torch.distributed as dist
    from moe_inference_verify_microbench_b200 import ops
    from moe_inference_verify_microbench_b200.hybrid import HybridBlock

    dev = _init(rank, world, port)
    try:
        H, I, E, k, nh, nkv, hd = 2048, 768, 128, 8, 32, 4, 128
        g = torch.Generator(device=dev)
        g.manual_seed(21)
        r = lambda *s, sc=0.02: (torch.randn(*s, generator=g, device=dev) * sc).to(torch.bfloat16)
        with torch.device(dev):
            blk = HybridBlock(H, I, nh, nkv, hd, E, k, world, rank, None, world, rank,
                              None).to(torch.bfloat16)
        wg, wu, wd = r(E, I, H), r(E, I, H), r(E, H, I)
        blk.weight_loader(1.0 + r(H, sc=0.1), r(nh * hd, H), r(nkv * hd, H), r(nkv * hd, H),
                          r(H, nh * hd), 1.0 + r(H, sc=0.1), r(E, H), list(wg), list(wu), list(wd))
        x = r(2, 64, H, sc=1.0)
        with torch.no_grad():
            y = blk(x)
            # the same block with the harness norms and the single-GPU layer
            h_ref = x + blk.attn(blk.attn_norm(x))
            n2 = blk.moe_norm(h_ref).reshape(-1, H).contiguous()
            y_ref = h_ref + ops.moe_layer(n2, blk.moe.gate.weight, wg, wu, wd, k).reshape(x.shape)
        torch.cuda.synchronize()
        ops.check_status(dev)
        err = ((y.float() - y_ref.float()).abs().amax(-1) /
               y_ref.float().abs().amax(-1)).reshape(-1).cpu()
        q.put((rank, float((err <= 2e-2).float().mean())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_hybrid_block_glue_matches_harness():
    """HybridBlock with the fused residual-add + RMSNorm row kernel against the
    harness norms + single-GPU layer (tp = ep = 1, one process)."""
    _need(1)
    res = _spawn(_block_worker, 1, (29960,))
    for rank, frac in res:
        assert frac >= 0.97, (rank, frac)  # a norm's last bit may flip a top-k boundary
