"""``bootcamp.ref.block.RMSNorm(hidden, eps)`` with a ``.weight`` parameter
(C8/python/solution.py:276,307): y = x / sqrt(mean(x^2) + eps) * weight,
computed in fp32 and cast back to the input dtype."""
import torch
from torch import nn


class RMSNorm(nn.Module):
    def __init__(self, hidden: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden))

    def forward(self, x):
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return (xf * r * self.weight.float()).to(x.dtype)
