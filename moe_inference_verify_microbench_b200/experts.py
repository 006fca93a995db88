"""Expert weight banks: stacked [E, I, H] / [E, H, I] storage behind
per-expert ``nn.Linear`` modules.

The reference keeps one ``SwiGLU_MLP`` per expert (C5/python/solution.py:68-80,
106) and loads weights by copying into ``experts[e].{gate,up,down}_proj.weight``
(C6/python/solution.py:98-110).  The grouped GEMMs want each projection as
one stacked tensor, so ``ExpertBank.bind`` packs the per-expert weights once
and re-points every expert's parameter at a view of the stack: later in-place
copies (``weight.data.copy_``, ``load_state_dict``) land in the stack with no
re-packing and no second copy of the 1.2 GB of expert weights.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


class SwiGLU_MLP(nn.Module):
    """``down_proj(silu(gate_proj(x)) * up_proj(x))``, bias-free
    (C5/python/solution.py:68-80)."""

    def __init__(self, hidden: int, intermediate: int):
        super().__init__()
        self.gate_proj = nn.Linear(in_features=hidden, out_features=intermediate, bias=False)
        self.up_proj = nn.Linear(in_features=hidden, out_features=intermediate, bias=False)
        self.down_proj = nn.Linear(in_features=intermediate, out_features=hidden, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class ExpertBank:
    """Stacked views of a ModuleList of ``SwiGLU_MLP`` experts."""

    def __init__(self) -> None:
        self.w_gate: torch.Tensor | None = None
        self.w_up: torch.Tensor | None = None
        self.w_down: torch.Tensor | None = None

    def invalidate(self) -> None:
        self.w_gate = self.w_up = self.w_down = None

    def _bound(self, experts: nn.ModuleList) -> bool:
        if self.w_gate is None or len(experts) == 0:
            return False
        for e in (0, len(experts) - 1):
            ex = experts[e]
            if (ex.gate_proj.weight.data_ptr() != self.w_gate[e].data_ptr()
                    or ex.up_proj.weight.data_ptr() != self.w_up[e].data_ptr()
                    or ex.down_proj.weight.data_ptr() != self.w_down[e].data_ptr()):
                return False
        return True

    @torch.no_grad()
    def bind(self, experts: nn.ModuleList):
        """Return (w_gate [E,I,H], w_up [E,I,H], w_down [E,H,I]), packing on first use."""
        if self._bound(experts):
            return self.w_gate, self.w_up, self.w_down
        E = len(experts)
        g0 = experts[0].gate_proj.weight
        I, H = g0.shape
        kw = dict(dtype=g0.dtype, device=g0.device)
        wg = torch.empty((E, I, H), **kw)
        wu = torch.empty((E, I, H), **kw)
        wd = torch.empty((E, H, I), **kw)
        for e, ex in enumerate(experts):
            wg[e].copy_(ex.gate_proj.weight)
            wu[e].copy_(ex.up_proj.weight)
            wd[e].copy_(ex.down_proj.weight)
            ex.gate_proj.weight.data = wg[e]
            ex.up_proj.weight.data = wu[e]
            ex.down_proj.weight.data = wd[e]
        self.w_gate, self.w_up, self.w_down = wg, wu, wd
        return wg, wu, wd


def router_bias_of(gate: nn.Linear) -> torch.Tensor | None:
    """fp32 router bias when the gate carries one (the skewed-routing
    workload swaps in an ``nn.Linear(bias=True)``); the reference gate has none."""
    b = getattr(gate, "bias", None)
    return None if b is None else b.detach().float().contiguous()


def qwen3_moe_layer_weights(state_dict, layer: int, num_experts: int,
                            prefix: str = "model.layers."):
    """One MoE layer's tensors from a Hugging Face Qwen3-MoE-style state dict
    (``{prefix}{layer}.mlp.gate.weight`` [E, H] and
    ``{prefix}{layer}.mlp.experts.{e}.{gate,up,down}_proj.weight``), returned as
    the argument lists of the reference's ``weight_loader``
    (C6/python/solution.py:98-110): ``(router, gate_list, up_list, down_list)``.
    ``state_dict`` only needs ``__getitem__`` (a dict, or a lazy mapping over
    checkpoint shards); nothing is copied here."""
    base = f"{prefix}{layer}.mlp."

    def get(name):
        try:
            return state_dict[base + name]
        except KeyError:
            raise KeyError(f"the state dict has no {base + name!r}") from None

    router = get("gate.weight")
    gate = [get(f"experts.{e}.gate_proj.weight") for e in range(num_experts)]
    up = [get(f"experts.{e}.up_proj.weight") for e in range(num_experts)]
    down = [get(f"experts.{e}.down_proj.weight") for e in range(num_experts)]
    return router, gate, up, down


@torch.no_grad()
def load_qwen3_moe_layer(module: nn.Module, state_dict, layer: int,
                         prefix: str = "model.layers.") -> None:
    """Copy one Qwen3-MoE layer of a checkpoint into a drop-in MoE module:
    ``PermutedSparseMoE`` (all experts), or an expert-parallel module
    (``EPSparseMoE`` lean / pure, ``HybridMoE``: the replicated router and this
    rank's expert shard, through its ``weight_loader``).  The expert weights
    land in the module's stacked [E, I, H] / [E, H, I] tensors, the layout the
    grouped GEMMs read, with no second copy.  Shapes are checked against the
    module before anything is copied."""
    E, H, I = module.num_experts, module.hidden, module.intermediate
    router, gate, up, down = qwen3_moe_layer_weights(state_dict, layer, E, prefix)
    want = [("gate.weight", router, (E, H))]
    for e in range(E):
        want += [(f"experts.{e}.gate_proj.weight", gate[e], (I, H)),
                 (f"experts.{e}.up_proj.weight", up[e], (I, H)),
                 (f"experts.{e}.down_proj.weight", down[e], (H, I))]
    for name, t, shape in want:
        if tuple(t.shape) != shape:
            raise ValueError(f"{prefix}{layer}.mlp.{name} has shape {tuple(t.shape)}, "
                             f"the module expects {shape}")
    if hasattr(module, "weight_loader"):
        module.weight_loader(router, gate, up, down)
        return
    module.gate.weight.copy_(router)
    wg, wu, wd = module.pack()
    for e in range(E):
        wg[e].copy_(gate[e])
        wu[e].copy_(up[e])
        wd[e].copy_(down[e])
