"""``PermutedSparseMoE`` — drop-in for C5/python/solution.py:82-161.

Same constructor, attributes (``gate``, ``experts[e].{gate,up,down}_proj``)
and forward contract (``[..., H] -> same shape``).  The forward is one C-ABI
call, ``moe_layer_forward``: router + top-k on tcgen05, a stable counting
sort, the row gather, the w13 grouped GEMM with SwiGLU fused, the w2 grouped
GEMM with the top-k weight fused, and a deterministic k-way combine.  It
issues no host synchronisation (the reference syncs once per expert on
``.item()``, C5:144).  The keyword extra ``index_add="atomic"`` switches the
un-permute to the reference's own semantics (index_add_, C5:160: fp32 atomic
accumulation per token, fused into the down GEMM).  With the keyword extra
``check_errors=True`` every forward synchronises and raises
``ops.MoEKernelError`` if a kernel reported a failure in the device status
word; by default the forward never synchronises and a failure is only
recorded there (``ops.check_status`` reads it).  With the keyword extra
``decode_weights=True`` the module also keeps the down weights transposed
(one more copy of ``w_down``; ``down_weights_transposed(refresh=True)``
rebuilds it after the per-expert weights were written) and runs batches of
up to 4 tokens on the one-pass decode layer.

The module must be bf16 on a CUDA device: there is no CPU path.
"""

from __future__ import annotations

import torch
from torch import nn

from . import ops
from .experts import ExpertBank, SwiGLU_MLP, router_bias_of

__all__ = ["PermutedSparseMoE", "SwiGLU_MLP"]


class PermutedSparseMoE(nn.Module):
    """Single-GPU sparse MoE with permutation + grouped compute (C5:82-161)."""

    def __init__(self, hidden: int, intermediate: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool = True, *, index_add: str = "deterministic",
                 check_errors: bool = False, decode_weights: bool = False) -> None:
        super().__init__()
        ops._combine_mode(index_add)  # validate
        self.index_add = index_add
        self.check_errors = check_errors
        self.decode_weights = decode_weights
        self._w_down_t = None
        self._w_down_t_key = None
        self.hidden = hidden
        self.intermediate = intermediate
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.gate = nn.Linear(hidden, num_experts, bias=False)
        self.experts = nn.ModuleList(SwiGLU_MLP(hidden, intermediate) for _ in range(num_experts))
        self._bank = ExpertBank()

    def _apply(self, fn, *args, **kwargs):
        self._bank.invalidate()
        self._w_down_t = None
        return super()._apply(fn, *args, **kwargs)

    def pack(self):
        """Stacked expert weights (w_gate, w_up, w_down), binding the per-expert
        parameters to views of them on first use."""
        return self._bank.bind(self.experts)

    def down_weights_transposed(self, refresh: bool = False) -> torch.Tensor:
        """w_down as [E, I, H] for the one-pass decode layer: built on first
        use and rebuilt when the stacked down weights are re-bound or written
        in place through the stacked tensor.  Writes through the per-expert
        parameters (``experts[e].down_proj.weight``) do not reach the stacked
        tensor's version counter: call with ``refresh=True`` after those."""
        wd = self.pack()[2]
        key = (wd.data_ptr(), wd._version)
        if refresh or self._w_down_t is None or self._w_down_t_key != key:
            self._w_down_t = ops.transpose_down_weights(wd)
            self._w_down_t_key = key
        return self._w_down_t

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x_flat = x.reshape(-1, shape[-1])
        if not x_flat.is_contiguous():
            x_flat = x_flat.contiguous()
        wg, wu, wd = self.pack()
        w_down_t = None
        if self.decode_weights and 0 < x_flat.shape[0] <= 4:
            w_down_t = self.down_weights_transposed()
        y = ops.moe_layer(x_flat, self.gate.weight, wg, wu, wd, self.top_k, self.norm_topk_prob,
                          bias=router_bias_of(self.gate), index_add=self.index_add,
                          w_down_t=w_down_t)
        if self.check_errors:
            ops.check_status(y.device)
        return y.reshape(shape)
