"""Build the sm_100a shared library ``libmoe_b200.so`` in-tree with nvcc.

    python -m moe_inference_verify_microbench_b200.build [--verbose]

The library exposes the C ABI declared in ``include/moe_b200.h``; the Python
package loads it with ctypes.  It links the CUDA runtime statically, so the
only runtime dependency is the NVIDIA driver.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libmoe_b200.so")
SOURCES = ["capi.cu", "gemm.cu", "sort_align.cu", "rows.cu", "sort_align_static.cu", "decode.cu",
           "ep_plan.cu", "ep_peer.cu"]
HEADERS = ["ptx.cuh", "grouped_gemm.cuh", "grouped_gemm_pair.cuh", "internal.h", "sort_block.cuh",
           "router_splitk.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, s) for s in SOURCES + HEADERS]
    files.append(os.path.join(REPO_DIR, "include", "moe_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every .cu under csrc/ for sm_100a and link ``libmoe_b200.so``."""
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    objdir = os.path.join(PKG_DIR, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    extra = ["-Xptxas", "-v"] if verbose else []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", os.path.join(REPO_DIR, "include"), "-c",
               os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force or a.verbose, verbose=a.verbose))


if __name__ == "__main__":
    main()
