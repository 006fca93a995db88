"""``all_to_all_variable`` — the variable-split all_to_all helper the
reference's expert-parallel schedules call (C7/python/solution.py:201,203,258,
C8 imports it at C8/python/solution.py:52); the reference imports it from a
module it does not ship, so its contract is taken from those call sites:
rows of ``x`` go out in ``input_split_sizes`` chunks (one per rank of
``group``) and the result holds ``sum(output_split_sizes)`` rows received in
rank order.  One NCCL all_to_all over NVLink."""

from __future__ import annotations

import torch
import torch.distributed as dist


def all_to_all_variable(x: torch.Tensor, input_split_sizes, output_split_sizes,
                        group: dist.ProcessGroup | None = None) -> torch.Tensor:
    in_splits = [int(v) for v in input_split_sizes]
    out_splits = [int(v) for v in output_split_sizes]
    if sum(in_splits) != x.shape[0]:
        raise ValueError(f"input splits sum to {sum(in_splits)}, x has {x.shape[0]} rows")
    out = torch.empty((sum(out_splits),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=group)
    return out
