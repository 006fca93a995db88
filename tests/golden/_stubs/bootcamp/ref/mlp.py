"""``bootcamp.ref.mlp.RefSwiGLU_MLP`` as its call sites use it
(C5/python/solution.py:66, C6/python/solution.py:95,108-110): three bias-free
projections named gate_proj / up_proj / down_proj, output
down(silu(gate(x)) * up(x))."""
import torch.nn.functional as F
from torch import nn


class RefSwiGLU_MLP(nn.Module):
    def __init__(self, hidden: int, intermediate: int) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(hidden, intermediate, bias=False)
        self.up_proj = nn.Linear(hidden, intermediate, bias=False)
        self.down_proj = nn.Linear(intermediate, hidden, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))
