"""The C ABI without a GPU: the library loads, exports exactly what
include/moe_b200.h declares, the bindings match, the host-only queries answer,
and the product path refuses CPU tensors (there is no CPU fallback)."""

import ctypes
import os
import re
import subprocess

import pytest
import torch

from moe_inference_verify_microbench_b200 import _native, ops

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "moe_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^MOE_API [^(]*?\b(moe_\w+)\(", text, flags=re.M)))


def test_library_loads_and_binds_every_declared_symbol():
    lib = _native.load()
    declared = header_functions()
    assert len(declared) >= 14
    assert sorted(_native.SIGNATURES) == declared
    for name in declared:
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_exported_dynamic_symbols_match_header():
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines() if " T moe_" in ln})
    assert exported == header_functions()


def test_host_queries():
    lib = _native.load()
    assert lib.moe_abi_version() == 5
    assert lib.moe_max_tiles(131072, 128) == 1024 + 128
    assert lib.moe_max_tiles(0, 16) == 16
    assert lib.moe_max_tiles_rows(131072, 128, 256) == 512 + 128
    assert lib.moe_max_tiles_rows(131072, 128, 128) == lib.moe_max_tiles(131072, 128)
    assert lib.moe_max_tiles_rows(1024, 16, 64) == 0  # only 128- and 256-row tiles
    assert lib.moe_layer_tile_rows(16384, 2048, 768, 128, 8) == 256  # CTA-pair GEMMs
    assert lib.moe_layer_tile_rows(4096, 2048, 768, 128, 8) == 128
    assert lib.moe_sort_align_workspace_bytes(8192, 128) >= 2 * 128 * 4
    ws = lib.moe_layer_workspace_bytes(16384, 2048, 768, 128, 8)
    assert ws >= 16384 * 8 * (768 + 2048) * 2  # h + weighted slot rows
    assert _native.error_string(-2) == "shape not supported by these kernels"
    assert "expert id" in _native.error_string(0x201)


def test_cpu_tensors_are_refused():
    x = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU path"):
        ops.router_topk(x, torch.zeros(16, 256, dtype=torch.bfloat16), 4)
    with pytest.raises(ValueError, match="no CPU path"):
        ops.sort_align(torch.zeros(8, dtype=torch.int32), 16)


def test_null_arguments_rejected_without_launch():
    lib = _native.load()
    # No device pointer is touched: argument checks run first on the host.
    assert lib.moe_layer_forward(None, None, None, None, None, None, 4, 256, 128, 16, 4, 1,
                                 None, 0, None, None, None) == -1
    assert lib.moe_sort_align(None, 8, 16, 0, 16, None, 0, None, None, None, None, None, None, 0,
                              None, None, None) == -1


def test_empty_batch_accepted_without_launch():
    """T, M or R = 0: every entry point returns 0 before any CUDA call, and the
    per-token buffers may be NULL (an empty torch tensor has no storage), as
    the reference's C5 forward accepts an empty batch; weights stay required
    and a positive count with a NULL buffer is still refused."""
    lib = _native.load()
    w = ctypes.c_void_p(256)  # stand-in weight / table address, never dereferenced
    H, I, E, k = 256, 128, 16, 4
    assert lib.moe_layer_forward(None, w, None, w, w, w, 0, H, I, E, k, 1, None, 0, None,
                                 None, None) == 0
    assert lib.moe_layer_forward_ex(None, w, None, w, w, w, 0, H, I, E, k, 1, 1, None, 0, None,
                                    None, None) == 0
    assert lib.moe_layer_forward(None, None, None, w, w, w, 0, H, I, E, k, 1, None, 0, None,
                                 None, None) == -1
    assert lib.moe_router_topk(None, w, None, 0, H, E, k, 1, None, None, None, None, None) == 0
    assert lib.moe_router_topk(None, w, None, 3, H, E, k, 1, None, None, None, None, None) == -1
    assert lib.moe_grouped_w13_swiglu(None, 0, w, w, E, w, w, E, H, I, None, None, None) == 0
    assert lib.moe_grouped_w13_swiglu(None, 5, w, w, E, w, w, E, H, I, None, None, None) == -1
    assert lib.moe_grouped_w13_swiglu_gather(None, 0, None, k, 0, w, w, E, w, w, E, H, I, None,
                                             None, None) == 0
    assert lib.moe_grouped_w2(None, 0, w, w, E, w, E, H, I, None, None, None, 0, None,
                              None) == 0
    assert lib.moe_grouped_w2(None, 0, w, w, E, None, E, H, I, None, None, None, 0, None,
                              None) == -1


def test_record_count_beyond_int32_is_refused_without_launch():
    """T * k routing records must fit the kernels' 32-bit record indices: a
    larger layer call returns MOE_RC_UNSUPPORTED before any pointer is used."""
    lib = _native.load()
    p = ctypes.c_void_p(256)  # stand-in addresses, never dereferenced
    T = (1 << 31) // 8        # T * 8 = 2^31 records: one past the int32 range
    assert lib.moe_layer_forward(p, p, None, p, p, p, T, 2048, 768, 128, 8, 1, p, 1 << 62, p,
                                 None, None) == -2
    assert lib.moe_layer_forward(p, p, None, p, p, p, T - 1, 2048, 768, 128, 8, 1, p, 0, p,
                                 None, None) == -5  # fits: then the workspace size is checked
    # the size query refuses the same shapes (0) instead of a wrapped size
    for mode in (0, 1):
        assert lib.moe_layer_workspace_bytes_ex(T, 2048, 768, 128, 8, mode) == 0
        assert lib.moe_layer_workspace_bytes_ex(T - 1, 2048, 768, 128, 8, mode) > 0
    assert lib.moe_layer_workspace_bytes(T, 2048, 768, 128, 8) == 0


def test_index_add_mode_is_validated():
    import torch
    from moe_inference_verify_microbench_b200 import PermutedSparseMoE, ops
    with pytest.raises(ValueError):
        PermutedSparseMoE(64, 32, 8, 2, index_add="sorted")
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.moe_layer(x, x, x, x, x, 2, index_add="fast")
    lib = ops._native.load()
    assert lib.moe_layer_workspace_bytes_ex(16, 2048, 768, 128, 8, 2) == 0
    # the atomic combine's fp32 token rows replace the bf16 slot rows
    assert (lib.moe_layer_workspace_bytes_ex(16384, 2048, 768, 128, 8, 1)
            < lib.moe_layer_workspace_bytes_ex(16384, 2048, 768, 128, 8, 0))
