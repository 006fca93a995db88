"""ctypes binding of ``libmoe_b200.so`` (the C ABI in ``include/moe_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every
op raises.  Build it with ``python -m moe_inference_verify_microbench_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmoe_b200.so")

_c_int = ctypes.c_int
_c_size = ctypes.c_size_t
_ptr = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/moe_b200.h one to one.
SIGNATURES: dict[str, tuple] = {
    "moe_abi_version": (_c_int, []),
    "moe_error_string": (ctypes.c_char_p, [_c_int]),
    "moe_router_topk": (_c_int, [_ptr, _ptr, _ptr, _c_int, _c_int, _c_int, _c_int, _c_int,
                                 _ptr, _ptr, _ptr, _ptr, _ptr]),
    "moe_sort_align_workspace_bytes": (_c_size, [_c_int, _c_int]),
    "moe_max_tiles": (_c_int, [_c_int, _c_int]),
    "moe_sort_align": (_c_int, [_ptr, _c_int, _c_int, _c_int, _c_int, _ptr, _c_size, _ptr, _ptr,
                                _ptr, _ptr, _ptr, _ptr, _c_int, _ptr, _ptr, _ptr]),
    "moe_sort_align_static_scratch": (_c_int, [_ptr, _c_int, _c_int, _c_int, _c_int, _ptr, _ptr,
                                               _ptr, _ptr, _ptr, _ptr, _c_int, _ptr, _ptr, _ptr]),
    "moe_tiles_from_offsets": (_c_int, [_ptr, _c_int, _ptr, _c_int, _ptr, _ptr, _ptr]),
    "moe_gather_rows": (_c_int, [_ptr, _c_int, _ptr, _c_int, _ptr, _c_int, _c_int, _ptr, _ptr,
                                 _ptr]),
    "moe_grouped_w13_swiglu": (_c_int, [_ptr, _c_int, _ptr, _ptr, _c_int, _ptr, _ptr, _c_int,
                                        _c_int, _c_int, _ptr, _ptr, _ptr]),
    "moe_grouped_w13_swiglu_gather": (_c_int, [_ptr, _c_int, _ptr, _c_int, _c_int, _ptr, _ptr,
                                               _c_int, _ptr, _ptr, _c_int, _c_int, _c_int, _ptr,
                                               _ptr, _ptr]),
    "moe_grouped_w2": (_c_int, [_ptr, _c_int, _ptr, _ptr, _c_int, _ptr, _c_int, _c_int, _c_int,
                                _ptr, _ptr, _ptr, _c_int, _ptr, _ptr]),
    "moe_combine": (_c_int, [_ptr, _c_int, _ptr, _ptr, _ptr, _c_int, _c_int, _c_int, _c_int,
                             _c_int, _ptr, _ptr, _ptr]),
    "moe_layer_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "moe_layer_forward": (_c_int, [_ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _c_int, _c_int, _c_int,
                                   _c_int, _c_int, _c_int, _ptr, _c_size, _ptr, _ptr, _ptr]),
    # ABI 2: tile tables of either height (128 or 256 rows)
    "moe_layer_tile_rows": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "moe_max_tiles_rows": (_c_int, [_c_int, _c_int, _c_int]),
    "moe_sort_align_rows": (_c_int, [_ptr, _c_int, _c_int, _c_int, _c_int, _ptr, _c_size, _ptr,
                                     _ptr, _ptr, _ptr, _ptr, _ptr, _c_int, _ptr, _c_int, _ptr,
                                     _ptr]),
    "moe_grouped_w13_swiglu_rows": (_c_int, [_ptr, _c_int, _ptr, _ptr, _c_int, _ptr, _ptr, _c_int,
                                             _c_int, _c_int, _ptr, _c_int, _ptr, _ptr]),
    "moe_grouped_w13_swiglu_gather_rows": (_c_int, [_ptr, _c_int, _ptr, _c_int, _c_int, _ptr,
                                                    _ptr, _c_int, _ptr, _ptr, _c_int, _c_int,
                                                    _c_int, _ptr, _c_int, _ptr, _ptr]),
    "moe_grouped_w2_rows": (_c_int, [_ptr, _c_int, _ptr, _ptr, _c_int, _ptr, _c_int, _c_int,
                                     _c_int, _ptr, _ptr, _ptr, _c_int, _c_int, _ptr, _ptr]),
    "moe_ep_keys": (_c_int, [_ptr, _c_int, _c_int, _c_int, _c_int, _ptr, _ptr, _ptr]),
    "moe_ep_meta": (_c_int, [_ptr, _ptr, _c_int, _ptr, _ptr, _c_int, _c_int, _c_int, _c_int,
                             _ptr, _ptr, _ptr]),
    # ABI 3: peer-store expert-parallel exchange
    "moe_ep_peer_buffer_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "moe_ep_peer_region_offset": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "moe_ep_peer_set_wait_limit_ms": (None, [_c_int]),
    "moe_ep_peer_alloc": (_c_int, [_c_size, _ptr, _ptr]),
    "moe_ep_peer_open": (_c_int, [_ptr, _ptr]),
    "moe_ep_peer_close": (_c_int, [_ptr]),
    "moe_ep_peer_free": (_c_int, [_ptr]),
    "moe_ep_peer_dispatch": (_c_int, [_ptr, _c_int, _c_int, _c_int, _c_int, _c_int, _ptr, _ptr,
                                      _c_int, _ptr, _ptr, _ptr, _c_int, _ptr, _ptr]),
    "moe_ep_peer_return": (_c_int, [_ptr, _c_int, _c_int, _c_int, _c_int, _c_int, _ptr, _c_int,
                                    _ptr, _ptr, _ptr]),
    # ABI 4: index_add_ semantics switch (atomic fp32 combine)
    "moe_layer_workspace_bytes_ex": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int]),
    "moe_layer_forward_ex": (_c_int, [_ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _c_int, _c_int, _c_int,
                                      _c_int, _c_int, _c_int, _c_int, _ptr, _c_size, _ptr, _ptr,
                                      _ptr]),
    "moe_grouped_w2_atomic_rows": (_c_int, [_ptr, _c_int, _ptr, _ptr, _c_int, _ptr, _c_int,
                                            _c_int, _c_int, _ptr, _ptr, _c_int, _c_int, _ptr,
                                            _c_int, _ptr, _ptr]),
    "moe_cast_f32_to_bf16": (_c_int, [_ptr, ctypes.c_longlong, _ptr, _ptr]),
    "moe_add_rmsnorm": (_c_int, [_ptr, _ptr, _ptr, _c_int, _c_int, ctypes.c_float, _ptr, _ptr,
                                 _ptr]),
    # ABI 5: SM budget for the grouped GEMMs
    "moe_device_sm_count": (_c_int, []),
    "moe_grouped_w13_swiglu_gather_ex": (_c_int, [_ptr, _c_int, _ptr, _c_int, _c_int, _ptr, _ptr,
                                                  _c_int, _ptr, _ptr, _c_int, _c_int, _c_int,
                                                  _ptr, _c_int, _c_int, _ptr, _ptr]),
    "moe_grouped_w2_ex": (_c_int, [_ptr, _c_int, _ptr, _ptr, _c_int, _ptr, _c_int, _c_int, _c_int,
                                   _ptr, _ptr, _ptr, _c_int, _c_int, _c_int, _ptr, _ptr]),
    # ABI 5: the one-pass decode layer on transposed down weights; last CUDA error
    "moe_decode_layer_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "moe_decode_layer_split": (_c_int, [_ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _c_int, _c_int, _c_int,
                                        _c_int, _c_int, _c_int, _ptr, _c_size, _ptr, _ptr, _ptr]),
    "moe_last_cuda_error": (_c_int, []),
}

ABI_VERSION = 5

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeLibraryError(RuntimeError):
    pass


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library and declare every exported signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise NativeLibraryError(
                f"{path} is missing; build it with `python -m moe_inference_verify_microbench_b200.build` "
                "(the CUDA path has no CPU fallback)")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.moe_abi_version() != ABI_VERSION:
            raise NativeLibraryError(f"ABI version mismatch: library {lib.moe_abi_version()}, "
                                     f"bindings {ABI_VERSION}")
        _lib = lib
        return lib


def error_string(code: int) -> str:
    return load().moe_error_string(int(code)).decode()
