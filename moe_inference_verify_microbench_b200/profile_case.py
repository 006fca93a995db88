"""A minimal MoE-layer workload for profilers (ncu launch lists and single
kernel captures): allocates only the layer's weights, input, output and
workspace, runs ``moe_layer_forward`` ``--steps`` times and checks the device
status word.

    python -m moe_inference_verify_microbench_b200.profile_case --tokens 4096 --steps 4
"""

from __future__ import annotations

import argparse

import torch

from . import ops

H, I, E, K = 2048, 768, 128, 8


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--steps", type=int, default=4)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    bf = torch.bfloat16
    x = torch.randn(a.tokens, H, generator=g, device=dev).to(bf)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(bf)
    ws = torch.empty(ops.layer_workspace_bytes(a.tokens, H, I, E, K), dtype=torch.uint8, device=dev)
    y = torch.empty_like(x)
    for _ in range(a.steps):
        ops.moe_layer(x, wr, wg, wu, wd, K, out=y, workspace=ws)
    torch.cuda.synchronize()
    ops.check_status(dev)
    print(f"profile_case ok: T={a.tokens} steps={a.steps} |y|max={y.abs().max().item():.4f}")


if __name__ == "__main__":
    main()
