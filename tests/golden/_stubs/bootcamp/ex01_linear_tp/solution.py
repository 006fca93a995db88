"""Alias: the reference's C1 component file, loaded from the reference
checkout named by the REFERENCE_ROOT environment variable."""
import importlib.util
import os
import sys

_p = os.path.join(os.environ["REFERENCE_ROOT"], "C1", "python", "solution.py")
_spec = importlib.util.spec_from_file_location("_ref_c1", _p)
_m = importlib.util.module_from_spec(_spec)
sys.modules["_ref_c1"] = _m
_spec.loader.exec_module(_m)
ColumnParallelLinear = _m.ColumnParallelLinear
RowParallelLinear = _m.RowParallelLinear
