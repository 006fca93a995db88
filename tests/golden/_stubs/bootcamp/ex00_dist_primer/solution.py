"""``all_to_all_variable(x, input_split_sizes, output_split_sizes, group)``
as its call sites use it (C7/python/solution.py:201,203,258): rows of ``x``
are sent in ``input_split_sizes`` chunks, one per rank, and the result holds
``sum(output_split_sizes)`` rows received in rank order."""
import torch
import torch.distributed as dist


def all_to_all_variable(x, input_split_sizes, output_split_sizes, group=None):
    out = torch.empty((int(sum(output_split_sizes)),) + tuple(x.shape[1:]),
                      dtype=x.dtype, device=x.device)
    dist.all_to_all_single(out, x.contiguous(), list(map(int, output_split_sizes)),
                           list(map(int, input_split_sizes)), group=group)
    return out
