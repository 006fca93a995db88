"""CPU restatement of the reference's single-device MoE forward in torch
(test and baseline infrastructure only: ``bench.py``'s ``cpu_baseline`` and
``--impl reference`` legs time it; the CUDA path never calls it).

The numpy oracle (``moe_oracle.py``) is the parity checker; its float64 /
numpy GEMMs run about ten times slower than the reference on the same CPU.
This module follows the same algorithm with the ops the reference itself uses
on a CPU, in bf16 torch, so its time stands for the reference's
(``oracle/calibrate_port.py`` measures the two against each other):

* router logits: one bf16 linear layer ........... C5/python/solution.py:124
* top-k of the logits, softmax of the k values
  (or of all E logits gathered at the k ids) ..... C5/python/solution.py:125-129
* records sorted by expert, per-expert counts .... C5/python/solution.py:131-134
* token rows gathered in expert order ............ C5/python/solution.py:135-137
* per expert: down(silu(gate(x)) * up(x)) ........ C5/python/solution.py:68-80, 142-157
* one weight scale, index_add_ into the output ... C5/python/solution.py:158-160

Weights are taken stacked ([E, I, H] gate and up, [E, H, I] down) instead of
per-expert modules; the sort is stable (the reference's is not, which only
reorders records inside an expert's block).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def permuted_moe_torch(x: torch.Tensor, router_weight: torch.Tensor, w_gate: torch.Tensor,
                       w_up: torch.Tensor, w_down: torch.Tensor, top_k: int,
                       norm_topk_prob: bool = True) -> torch.Tensor:
    """y [N, H] for x [N, H]; every tensor bf16 on the CPU."""
    n_tok = x.shape[0]
    num_experts = router_weight.shape[0]
    logits = F.linear(x, router_weight)
    top_vals, top_ids = torch.topk(logits, top_k, dim=-1)
    if norm_topk_prob:
        weights = F.softmax(top_vals, dim=-1)
    else:
        weights = F.softmax(logits, dim=-1).gather(-1, top_ids)
    flat_ids = top_ids.reshape(-1)
    order = torch.argsort(flat_ids, stable=True)
    counts = torch.bincount(flat_ids, minlength=num_experts).tolist()
    token_of = order // top_k
    rows = x[token_of]
    out = torch.empty_like(rows)
    begin = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        seg = rows[begin:begin + c]
        act = F.silu(F.linear(seg, w_gate[e])) * F.linear(seg, w_up[e])
        out[begin:begin + c] = F.linear(act, w_down[e])
        begin += c
    out *= weights.reshape(-1)[order][:, None]
    y = torch.zeros_like(x)
    y.index_add_(0, token_of, out)
    return y
