"""Shared test helpers: seeded inputs, bf16 conversions, oracle adapters."""

from __future__ import annotations

import os

import numpy as np
import torch

from oracle import moe_oracle as mo

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Output tolerance: max|y - y_ref| / max|y_ref| against the fp32 oracle.
REL_TOL = 2e-2


def to_t(bits: np.ndarray, device=None) -> torch.Tensor:
    """uint16 bf16 bits -> bf16 torch tensor."""
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)
    return t.to(device) if device is not None else t


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def inputs(T, H, I, E, seed=0, device=None):
    d = mo.make_inputs(T, H, I, E, seed)
    f = {k: mo.f32_from_bf16_bits(v) for k, v in d.items()}
    t = {k: to_t(v, device) for k, v in d.items()} if device is not None else None
    return f, t


def ragged_counts(E, total, rng, empty_frac=0.25):
    """Per-expert counts summing to `total` with some empty experts."""
    w = rng.random(E)
    w[rng.random(E) < empty_frac] = 0.0
    if w.sum() == 0:
        w[0] = 1.0
    c = np.floor(w / w.sum() * total).astype(np.int64)
    c[np.argmax(w)] += total - c.sum()
    return c


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def sample_token_outputs(xf, wg, wu, wd, ids, w, tokens):
    """fp32 oracle output for selected tokens given routing (ids, weights)."""
    out = np.zeros((len(tokens), xf.shape[1]), dtype=np.float32)
    for i, n in enumerate(tokens):
        for j in range(ids.shape[1]):
            e = int(ids[n, j])
            o = mo.swiglu_expert(xf[n:n + 1], wg[e], wu[e], wd[e], mode="fp32")
            out[i] += w[n, j] * o[0]
    return out
