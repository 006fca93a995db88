"""``build_rope_cache(T, head_dim, base, device, dtype) -> (cos, sin)`` and
``apply_rope(x[B,T,h,d], cos, sin)`` as C4/python/solution.py:260-264 call
them.  The reference does not pin the rotation convention; this uses the
half-split (rotate_half) form."""
import torch


def build_rope_cache(T, head_dim, base=10000.0, device=None, dtype=torch.float32):
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    t = torch.arange(T, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    d = x.shape[-1]
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    return (x.float() * c.float() + rot.float() * s.float()).to(x.dtype)
