"""Time the CPU restatements of C5 against the unmodified reference C5 on the
same CPU, the same sample and the same thread count (test infrastructure;
runs only where the reference checkout is present).

The GPU box has no copy of the reference, so ``bench.py --impl reference``
and ``cpu_baseline`` time a restatement (``kind: "port"``): the torch port
(``moe_torch_port.py``).  This script measures how its speed, and the numpy
oracle's, compare with the reference's own CPU path
(C5/python/solution.py:108-161, loaded with the helper stand-ins of
``tests/golden/_stubs``), so the port's numbers can be read as the
reference's, and checks that the torch port's output equals the reference's:

    REFERENCE_ROOT=<reference checkout> python oracle/calibrate_port.py [--tokens 256] [--reps 3]

It prints one JSON line: the three times, their ratios to the reference,
the thread count and the torch port's largest difference from the reference
output.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import platform
import statistics
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests", "golden", "_stubs"))

from oracle import moe_oracle as mo  # noqa: E402
from oracle.moe_torch_port import permuted_moe_torch  # noqa: E402


def load_c5(root: str):
    path = os.path.join(root, "C5", "python", "solution.py")
    spec = importlib.util.spec_from_file_location("_ref_c5_calibrate", path)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    root = os.environ.get("REFERENCE_ROOT")
    if not root or not os.path.isdir(root):
        sys.exit("set REFERENCE_ROOT to the reference checkout (the directory holding C5/)")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    T, H, I, E, k = args.tokens, 2048, 768, 128, 8
    inp = mo.make_inputs(T, H, I, E, 0)
    f = {n: mo.f32_from_bf16_bits(v) for n, v in inp.items()}
    bf = {n: torch.from_numpy(v).to(torch.bfloat16) for n, v in f.items()}

    c5 = load_c5(root)
    mod = c5.PermutedSparseMoE(H, I, E, k).to(torch.bfloat16)
    with torch.no_grad():
        mod.gate.weight.copy_(bf["wr"])
        for e, ex in enumerate(mod.experts):
            ex.gate_proj.weight.copy_(bf["w_gate"][e])
            ex.up_proj.weight.copy_(bf["w_up"][e])
            ex.down_proj.weight.copy_(bf["w_down"][e])

    def time_it(fn):
        fn()  # warm-up
        ts = []
        for _ in range(args.reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    with torch.no_grad():
        t_ref = time_it(lambda: mod(bf["x"]))
        t_torch = time_it(lambda: permuted_moe_torch(bf["x"], bf["wr"], bf["w_gate"], bf["w_up"],
                                                     bf["w_down"], k))
        y_ref = mod(bf["x"]).float()
        y_torch = permuted_moe_torch(bf["x"], bf["wr"], bf["w_gate"], bf["w_up"], bf["w_down"],
                                     k).float()
    t_numpy = time_it(lambda: mo.permuted_moe(f["x"], f["wr"], f["w_gate"], f["w_up"],
                                              f["w_down"], k, True, mode="ref"))
    print(json.dumps({
        "tokens": T, "threads": threads, "cpu": platform.processor() or platform.machine(),
        "reference_c5_s": t_ref, "torch_port_s": t_torch, "numpy_oracle_s": t_numpy,
        "reference_tokens_per_s": T / t_ref, "torch_port_tokens_per_s": T / t_torch,
        "numpy_oracle_tokens_per_s": T / t_numpy,
        "torch_port_over_reference_speed": t_ref / t_torch,
        "numpy_oracle_over_reference_speed": t_ref / t_numpy,
        "torch_port_max_rel_diff": float((y_torch - y_ref).abs().max() / y_ref.abs().max()),
    }))


if __name__ == "__main__":
    main()
