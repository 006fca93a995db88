"""Small profiling case for the one-pass decode layer (one B200): builds
seeded Qwen3-30B-A3B MoE weights and their transposed down copy, runs
``decode_layer_split`` ``--steps`` times at ``--tokens`` tokens and checks the
status word.  Meant to run under ``ncu`` (a few hundred MB on the device).

    python -m moe_inference_verify_microbench_b200.profile_decode --tokens 1 --steps 3
"""

from __future__ import annotations

import argparse

import torch

from . import ops

H, I, E, K = 2048, 768, 128, 8


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    bf = torch.bfloat16
    r = lambda *s, sc=0.02: (torch.randn(*s, generator=g, device=dev) * sc).to(bf)  # noqa: E731
    wr, wg, wu, wd = r(E, H), r(E, I, H), r(E, I, H), r(E, H, I)
    wdt = ops.transpose_down_weights(wd)
    x = r(a.tokens, H, sc=1.0)
    ws = torch.empty(ops.decode_layer_workspace_bytes(a.tokens, H, E), dtype=torch.uint8, device=dev)
    y = torch.empty_like(x)
    for _ in range(a.steps):
        ops.decode_layer_split(x, wr, wg, wu, wdt, K, out=y, workspace=ws)
    torch.cuda.synchronize()
    ops.check_status(dev)
    print(f"profile_decode ok: T={a.tokens} steps={a.steps} |y|max={y.abs().max().item():.4f}")


if __name__ == "__main__":
    main()
