"""C6 drop-in: ``EPSparseMoE`` with the lean single-all_reduce schedule
(C6/python/solution.py:57-182)."""

from .ep import EPSparseMoELean as EPSparseMoE

__all__ = ["EPSparseMoE"]
