"""Generate the golden fixtures in this directory by running the reference
suite itself (weidotwisc/moe_inference_verify_microbench) on CPU.

Run in a container that has the reference checkout:

    REFERENCE_ROOT=<path of the reference checkout> python tests/golden/make_golden.py

The reference imports helper modules it does not ship; ``_stubs/bootcamp``
provides them, restated from their call sites.  Inputs come from
``oracle.moe_oracle.make_inputs`` (numpy PCG64, reproducible on any host), so
fixtures for the full-size shapes store only outputs.

Fixtures written:

* ``c5_small_s{0,1}.npz``   C5 PermutedSparseMoE, T=64 H=128 I=64 E=16 k=4, inputs + outputs
* ``c5_small_nonorm.npz``   same, ``norm_topk_prob=False``
* ``c5_full_t256.npz``      C5 at H=2048 I=768 E=128 k=8, T=256, seed 0 (outputs only)
* ``c9_fp32.npz``           C9 fused_moe_forward under the Triton CPU interpreter in
                            fp32 (bf16 is wrong under the interpreter), ragged and
                            empty experts
* ``ep_{c6,c7,c8}_*.npz``   C6 / C7 / C8-HybridMoE on 2, 4 and 8 gloo ranks (C7 also with
                            the Zipf router skew, C8 at tp=2 and tp=4); per-rank outputs
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("REFERENCE_ROOT")
if not REF or not os.path.isdir(REF):
    sys.exit("set REFERENCE_ROOT to the reference checkout (the directory holding C5/ ... C9/)")
sys.path.insert(0, os.path.join(HERE, "_stubs"))
sys.path.insert(0, REPO)

from oracle import moe_oracle as mo  # noqa: E402


def load_ref(component: str, name: str):
    path = os.path.join(REF, component, "python", "solution.py")
    spec = importlib.util.spec_from_file_location(name, path)
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


def t_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(mo.f32_from_bf16_bits(bits)).to(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def load_c5_weights(mod, inp):
    mod.gate.weight.data.copy_(t_bf16(inp["wr"]))
    for e, ex in enumerate(mod.experts):
        ex.gate_proj.weight.data.copy_(t_bf16(inp["w_gate"][e]))
        ex.up_proj.weight.data.copy_(t_bf16(inp["w_up"][e]))
        ex.down_proj.weight.data.copy_(t_bf16(inp["w_down"][e]))


def run_c5(T, H, I, E, k, seed, norm=True, store_inputs=True):
    c5 = load_ref("C5", "_ref_c5")
    inp = mo.make_inputs(T, H, I, E, seed)
    mod = c5.PermutedSparseMoE(H, I, E, k, norm_topk_prob=norm).to(torch.bfloat16)
    load_c5_weights(mod, inp)
    x = t_bf16(inp["x"])
    with torch.no_grad():
        logits = mod.gate(x)
        tv, ti = torch.topk(logits, k, dim=-1)
        sv, si = torch.sort(logits, dim=-1, descending=True, stable=True)
        y = mod(x)
    out = dict(T=T, H=H, I=I, E=E, k=k, seed=seed, norm=int(norm),
               logits=bits(logits), topk_vals=bits(tv), topk_ids=ti.numpy(),
               stable_ids=si[:, :k].numpy(), y=bits(y))
    if store_inputs:
        out.update(inp)
    return out


def run_c9_fp32():
    os.environ["TRITON_INTERPRET"] = "1"
    c9 = load_ref("C9", "_ref_c9")
    rng = np.random.default_rng(7)
    H, I, E = 96, 80, 6
    counts = np.array([5, 0, 64, 1, 0, 70], dtype=np.int64)  # empty, single, >BLOCK_M
    offsets = np.zeros(E + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    M = int(offsets[-1])
    sx = rng.standard_normal((M, H), dtype=np.float32)
    wg = rng.standard_normal((E, I, H), dtype=np.float32) * 0.05
    wu = rng.standard_normal((E, I, H), dtype=np.float32) * 0.05
    wd = rng.standard_normal((E, H, I), dtype=np.float32) * 0.05
    y = c9.fused_moe_forward(torch.from_numpy(sx), torch.from_numpy(offsets), torch.from_numpy(wg),
                             torch.from_numpy(wu), torch.from_numpy(wd))
    return dict(sorted_x=sx, offsets=offsets, w_gate=wg, w_up=wu, w_down=wd, y=y.numpy())


# ---------------------------------------------------------------------------
# Expert-parallel schedules on gloo ranks
# ---------------------------------------------------------------------------

EP_SHAPE = dict(T=64, H=128, I=64, E=16, k=4)


def _ep_worker(rank, world, port, kind, ep, tp, seed, zipf, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, os.path.join(HERE, "_stubs"))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    s = EP_SHAPE
    T, H, I, E, k = s["T"], s["H"], s["I"], s["E"], s["k"]
    inp = mo.make_inputs(T * world, H, I, E, seed)
    xall = t_bf16(inp["x"])
    wr = t_bf16(inp["wr"])
    wg = [t_bf16(inp["w_gate"][e]) for e in range(E)]
    wu = [t_bf16(inp["w_up"][e]) for e in range(E)]
    wd = [t_bf16(inp["w_down"][e]) for e in range(E)]
    bias = torch.from_numpy(mo.zipf_bias(E)) if zipf else None
    with torch.no_grad():
        if kind == "c6":
            m = load_ref("C6", "_ref_c6")
            mod = m.EPSparseMoE(H, I, E, k, ep, rank, group=None).to(torch.bfloat16)
            mod.weight_loader(wr, wg, wu, wd)
            x = xall[:T]  # replicated input: every rank holds the same T tokens
        elif kind == "c7":
            m = load_ref("C7", "_ref_c7")
            mod = m.EPSparseMoE(H, I, E, k, ep, rank, group=None).to(torch.bfloat16)
            mod.weight_loader(wr, wg, wu, wd)
            x = xall[rank * T:(rank + 1) * T]  # distinct tokens per rank
        else:
            m = load_ref("C8", "_ref_c8")
            dp = world // tp
            tp_groups = [dist.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(dp)]
            tg = tp_groups[rank // tp]
            mod = m.HybridMoE(H, I, E, k, tp, rank % tp, tg, ep, rank, None).to(torch.bfloat16)
            mod.weight_loader(wr, wg, wu, wd)
            g = rank // tp  # DP index: each TP group holds its own T tokens, replicated inside
            x = xall[g * T:(g + 1) * T]
        if bias is not None:
            lin = torch.nn.Linear(H, E, bias=True).to(torch.bfloat16)
            lin.weight.data.copy_(wr)
            lin.bias.data.copy_(bias.to(torch.bfloat16))
            mod.gate = lin
        y = mod(x)
    q.put((rank, bits(y)))
    dist.barrier()
    dist.destroy_process_group()


def run_ep(kind, world, tp=1, seed=0, zipf=False, port=29611):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, kind, world, tp, seed, zipf, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    s = EP_SHAPE
    out = dict(kind=kind, world=world, tp=tp, seed=seed, zipf=int(zipf), **s)
    for r in range(world):
        out[f"y_rank{r}"] = res[r]
    return out


FIXTURES = {
    "c5_small_s0.npz": lambda: run_c5(64, 128, 64, 16, 4, seed=0),
    "c5_small_s1.npz": lambda: run_c5(64, 128, 64, 16, 4, seed=1),
    "c5_small_nonorm.npz": lambda: run_c5(64, 128, 64, 16, 4, seed=2, norm=False),
    "c5_full_t256.npz": lambda: run_c5(256, 2048, 768, 128, 8, seed=0, store_inputs=False),
    "c9_fp32.npz": run_c9_fp32,
    "ep_c6_w2.npz": lambda: run_ep("c6", 2, port=29611),
    "ep_c6_w4.npz": lambda: run_ep("c6", 4, port=29612),
    "ep_c7_w2.npz": lambda: run_ep("c7", 2, port=29613),
    "ep_c7_w4_zipf.npz": lambda: run_ep("c7", 4, zipf=True, port=29614),
    "ep_c8_w4_tp2.npz": lambda: run_ep("c8", 4, tp=2, port=29615),
    # eight ranks: the expert-parallel configurations at their own world size
    # (C6 ep=8; C7 dp=ep=8 with the Zipf router skew; C8 tp=2 x dp=4 and tp=4 x dp=2)
    "ep_c6_w8.npz": lambda: run_ep("c6", 8, port=29616),
    "ep_c7_w8_zipf.npz": lambda: run_ep("c7", 8, zipf=True, port=29617),
    "ep_c8_w8_tp2.npz": lambda: run_ep("c8", 8, tp=2, port=29618),
    "ep_c8_w8_tp4.npz": lambda: run_ep("c8", 8, tp=4, port=29619),
}


def main():
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*", default=None,
                    help="fixture file names to (re)write; default: all")
    names = ap.parse_args().only or list(FIXTURES)
    unknown = sorted(set(names) - set(FIXTURES))
    if unknown:
        sys.exit(f"unknown fixtures {unknown}; known: {sorted(FIXTURES)}")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name in names:
        np.savez_compressed(os.path.join(HERE, name), **FIXTURES[name]())
        print("wrote", name, flush=True)


if __name__ == "__main__":
    main()
