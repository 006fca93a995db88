"""C7 drop-in: ``EPSparseMoE`` with the all_to_all dispatch/combine schedule
(C7/python/solution.py:65-269)."""

from .ep import EPSparseMoEPure as EPSparseMoE

__all__ = ["EPSparseMoE"]
