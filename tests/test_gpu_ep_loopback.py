"""Expert-parallel schedules on ONE GPU: every rank is a thread of this process
running the real CUDA kernels of its shard, with the collectives emulated by
device copies (``loopback.LoopbackWorld``).  This checks the GPU path of C6
(EPSparseMoE lean, C6/python/solution.py:112-182), C7 (EPSparseMoE pure,
C7/python/solution.py:120-269) and C8 (HybridMoE, C8/python/solution.py:
139-230) at 2, 4 and 8 ranks where only one GPU is available:

* at the fixture shapes, against the reference's own per-rank outputs
  (tests/golden/ep_*.npz, made by the unmodified reference on gloo ranks);
* at the expert-parallel configurations' own shapes (H=2048, I=768, E=128,
  top-8: C6 ep=8 on 4096 replicated tokens; C7 dp=ep=8 on 2048 tokens per
  rank with the Zipf router skew; C8 on 8 x 2048 tokens at tp=2 x dp=4 and
  tp=4 x dp=2), against the single-GPU layer on the same tokens and against
  an fp32 evaluation of sampled tokens.

The NCCL transport is used (host-synchronised splits); the peer-store
transport's kernels wait on one another and cannot share a GPU."""

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8


def _build(kind, world, rank, tp, Hh, Ii, Ee, k, wr, wg, wu, wd, bias, dev, dist):
    from moe_inference_verify_microbench_b200.ep_lean import EPSparseMoE as Lean
    from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE as Pure
    from moe_inference_verify_microbench_b200.hybrid import HybridMoE
    with torch.device(dev):
        if kind == "c6":
            mod = Lean(Hh, Ii, Ee, k, world, rank, group=None)
        elif kind == "c7":
            mod = Pure(Hh, Ii, Ee, k, world, rank, group=None, transport="nccl")
        else:
            groups = [dist.new_group(list(range(i * tp, (i + 1) * tp))) for i in range(world // tp)]
            mod = HybridMoE(Hh, Ii, Ee, k, tp, rank % tp, groups[rank // tp], world, rank, None,
                            transport="nccl")
        mod = mod.to(torch.bfloat16)
    mod.weight_loader(wr, wg, wu, wd)
    if bias is not None:
        lin = torch.nn.Linear(Hh, Ee, bias=True).to(torch.bfloat16).to(dev)
        lin.weight.data.copy_(wr)
        lin.bias.data.copy_(bias)
        mod.gate = lin
    return mod


def _rank_tokens(kind, world, rank, tp, T):
    """Rows of the job's input that rank `rank` is given (C6: all T replicated;
    C7: its own T; C8: the T tokens of its TP group)."""
    if kind == "c6":
        return slice(0, T)
    if kind == "c7":
        return slice(rank * T, (rank + 1) * T)
    g = rank // tp
    return slice(g * T, (g + 1) * T)


FIXTURES = [("ep_c6_w2.npz", 2), ("ep_c6_w4.npz", 4), ("ep_c6_w8.npz", 8), ("ep_c7_w2.npz", 2),
            ("ep_c7_w4_zipf.npz", 4), ("ep_c7_w8_zipf.npz", 8), ("ep_c8_w4_tp2.npz", 4),
            ("ep_c8_w8_tp2.npz", 8), ("ep_c8_w8_tp4.npz", 8)]


@pytest.mark.parametrize("name,world", FIXTURES)
def test_ep_schedule_loopback_matches_reference(cuda, name, world):
    import torch.distributed as dist
    from helpers import load_golden, to_t
    from loopback import LoopbackWorld
    from moe_inference_verify_microbench_b200 import ops
    from oracle import moe_oracle as mo

    dev = cuda
    g = load_golden(name)
    T, Hh, Ii, Ee, k, tp = (int(g[n]) for n in ("T", "H", "I", "E", "k", "tp"))
    kind = str(g["kind"])
    d = mo.make_inputs(T * world, Hh, Ii, Ee, int(g["seed"]))
    xall = to_t(d["x"], dev)
    wr = to_t(d["wr"], dev)
    wg, wu, wd = (to_t(d[n], dev) for n in ("w_gate", "w_up", "w_down"))
    bias = (torch.from_numpy(mo.zipf_bias(Ee)).to(torch.bfloat16).to(dev)
            if int(g["zipf"]) else None)
    lw = LoopbackWorld(world, dev)

    def rank_fn(rank):
        mod = _build(kind, world, rank, tp, Hh, Ii, Ee, k, wr, wg, wu, wd, bias, dev, dist)
        x = xall[_rank_tokens(kind, world, rank, tp, T)].contiguous()
        with torch.no_grad():
            y = mod(x)
        return x, y

    out = lw.run(rank_fn)
    torch.cuda.synchronize()
    ops.check_status(dev)
    for rank, (x, y) in enumerate(out):
        _, _, lg = ops.router_topk(x, wr, k, bias=None if bias is None else bias.float(),
                                   return_logits=True)
        srt = torch.sort(lg.float(), dim=-1, descending=True).values
        tie = (srt[:, k - 1] == srt[:, k]).cpu().numpy()
        yref = mo.f32_from_bf16_bits(g[f"y_rank{rank}"])
        assert tie.mean() <= 0.2, (rank, tie.mean())
        err = mo.rel_err(y.float().cpu().numpy()[~tie], yref[~tie])
        assert err <= 2e-2, (name, rank, err)


def _fp32_tokens(x, ids, w, wg, wu, wd, tokens):
    """fp32 evaluation of the MoE output of the given tokens from their routing
    (C5/python/solution.py:142-160 without intermediate bf16 rounding)."""
    out = []
    for n in tokens:
        acc = torch.zeros(x.shape[1], dtype=torch.float32, device=x.device)
        xn = x[n].float()
        for j in range(ids.shape[1]):
            e = int(ids[n, j])
            h = torch.nn.functional.silu(wg[e].float() @ xn) * (wu[e].float() @ xn)
            acc += w[n, j].float() * (wd[e].float() @ h)
        out.append(acc)
    return torch.stack(out)


def _config_inputs(dev, T_all, seed=0):
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    bf = torch.bfloat16
    x = torch.randn(T_all, H, generator=gen, device=dev).to(bf)
    wr = (torch.randn(E, H, generator=gen, device=dev) * 0.02).to(bf)
    wg = (torch.randn(E, I, H, generator=gen, device=dev) * 0.02).to(bf)
    wu = (torch.randn(E, I, H, generator=gen, device=dev) * 0.02).to(bf)
    wd = (torch.randn(E, H, I, generator=gen, device=dev) * 0.02).to(bf)
    return x, wr, wg, wu, wd


@pytest.mark.parametrize("kind,world,tp,T,zipf", [
    ("c6", 8, 1, 4096, False),     # C6: ep=8, 4096 tokens replicated on every rank
    ("c7", 8, 1, 2048, True),      # C7: dp=ep=8, 2048 tokens per rank, Zipf(1.2) router skew
    ("c8", 8, 2, 4096, False),     # C8: 8 x 2048 tokens, tp=2 x dp=4 (4096 per TP group)
    ("c8", 8, 4, 8192, False),     # C8: tp=4 x dp=2 (8192 per TP group)
])
def test_ep_config_shapes_loopback(cuda, kind, world, tp, T, zipf):
    import torch.distributed as dist
    from loopback import LoopbackWorld
    from moe_inference_verify_microbench_b200 import ops
    from oracle import moe_oracle as mo

    dev = cuda
    groups = 1 if kind == "c6" else (world if kind == "c7" else world // tp)
    T_all = T * groups
    x, wr, wg, wu, wd = _config_inputs(dev, T_all)
    bias = torch.from_numpy(mo.zipf_bias(E)).to(torch.bfloat16).to(dev) if zipf else None
    bias32 = None if bias is None else bias.float()
    lw = LoopbackWorld(world, dev)

    def rank_fn(rank):
        mod = _build(kind, world, rank, tp, H, I, E, K, wr, wg, wu, wd, bias, dev, dist)
        xs = x[_rank_tokens(kind, world, rank, tp, T)].contiguous()
        with torch.no_grad():
            y = mod(xs)
        del mod
        return y

    ys = lw.run(rank_fn)
    torch.cuda.synchronize()
    ops.check_status(dev)
    # The whole job on the single-GPU layer (itself pinned to the oracle).
    y1 = ops.moe_layer(x, wr, wg, wu, wd, K, bias=bias32)
    ids, w, _ = ops.router_topk(x, wr, K, bias=bias32)
    if zipf:  # the skew concentrates the load on the low expert ids
        counts = torch.bincount(ids.reshape(-1).long(), minlength=E).float()
        assert counts[:E // world].sum() > 2 * counts[-E // world:].sum()
    ref = y1.float()
    scale = ref.abs().max()
    rng = np.random.default_rng(0)
    for rank, y in enumerate(ys):
        sl = _rank_tokens(kind, world, rank, tp, T)
        assert y.shape == (sl.stop - sl.start, H)
        err = ((y.float() - ref[sl]).abs().max() / scale).item()
        assert err <= 1e-2, (kind, rank, err)
    # Sampled tokens of rank 0 and of the last rank against an fp32 evaluation.
    for rank in (0, world - 1):
        sl = _rank_tokens(kind, world, rank, tp, T)
        toks = sorted(rng.choice(sl.stop - sl.start, size=12, replace=False).tolist())
        glob = [sl.start + t for t in toks]
        yf = _fp32_tokens(x, ids, w, wg, wu, wd, glob)
        err = ((ys[rank][toks].float() - yf).abs().max() / yf.abs().max()).item()
        assert err <= 2e-2, (kind, rank, err)
