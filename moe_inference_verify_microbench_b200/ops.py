"""Torch-tensor wrappers over the C ABI (``include/moe_b200.h``).

Each op checks devices, dtypes and contiguity, allocates its outputs with the
torch caching allocator, and launches on the current CUDA stream.  Nothing
here synchronises the host; device-side errors land in a per-device status
word that ``check_status`` reads (tests and debugging only).
"""

from __future__ import annotations

import ctypes
from typing import NamedTuple

import torch

from . import _native

BLOCK_M = 128


class MoEKernelError(RuntimeError):
    """A C-ABI call refused its arguments (``code`` < 0, a MOE_RC_* value) or a
    kernel reported a failure in the device status word (``code`` > 0, a
    MOE_ERR_* value)."""

    def __init__(self, message: str, code: int = 0) -> None:
        super().__init__(message)
        self.code = code


ERR_PEER_TIMEOUT = 0x105  # MOE_ERR_PEER_TIMEOUT
RC_UNSUPPORTED = -2       # MOE_RC_UNSUPPORTED


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The int32 device status word the kernels of ``device`` report into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Synchronise and raise ``MoEKernelError`` if any kernel on ``device``
    reported an error (then the word is cleared unless ``reset`` is False).
    The modules call this after every forward when built with
    ``check_errors=True``; otherwise a device-side failure (an expert id out of
    range, a bounded wait that ran out) is only recorded, and the forward's
    output is not to be trusted until the caller has checked."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    st = status_word(device)
    code = int(st.item())
    if reset and code:
        st.zero_()
    if code:
        raise MoEKernelError(f"device status 0x{code:x}: {_native.error_string(code)}", code)


def _p(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need(t: torch.Tensor, name: str, dtype: torch.dtype, ndim: int | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor: the MoE kernels have no CPU path")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _rc(rc: int, what: str) -> None:
    if rc != 0:
        raise MoEKernelError(f"{what}: {_native.error_string(rc)} (rc={rc})", rc)


# --------------------------------------------------------------------------- router


def router_topk(x: torch.Tensor, router_weight: torch.Tensor, top_k: int,
                norm_topk_prob: bool = True, bias: torch.Tensor | None = None,
                return_logits: bool = False):
    """Router GEMM + top-k + softmax (C5/python/solution.py:124-129).

    Returns (ids int32 [T,k], weights fp32 [T,k], logits bf16 [T,E] or None).
    """
    _need(x, "x", torch.bfloat16, 2)
    _need(router_weight, "router_weight", torch.bfloat16, 2)
    T, H = x.shape
    E = router_weight.shape[0]
    if router_weight.shape[1] != H:
        raise ValueError("router_weight must be [E, H]")
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    dev = x.device
    ids = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, top_k), dtype=torch.float32, device=dev)
    logits = torch.empty((T, E), dtype=torch.bfloat16, device=dev) if return_logits else None
    lib = _native.load()
    _rc(lib.moe_router_topk(_p(x), _p(router_weight), _p(bias), T, H, E, top_k,
                            int(bool(norm_topk_prob)), _p(ids), _p(w), _p(logits),
                            _p(status_word(dev)), _stream(dev)), "moe_router_topk")
    return ids, w, logits


# --------------------------------------------------------------------------- sort / align


class SortResult(NamedTuple):
    counts: torch.Tensor      # int32 [E_local]
    offsets: torch.Tensor     # int32 [E_local + 1]
    offsets64: torch.Tensor | None  # int64 [E_local + 1]
    perm: torch.Tensor        # int32 [R]; valid below offsets[E_local]
    inv: torch.Tensor | None  # int32 [R]; -1 for records outside the expert range
    tiles: torch.Tensor       # int32 [max_tiles, 4]
    num_tiles: torch.Tensor   # int32 [1]
    max_tiles: int
    tile_rows: int = 128      # height of the tile table's row blocks (128 or 256)


def max_tiles(R: int, e_local: int, tile_rows: int = 128) -> int:
    return int(_native.load().moe_max_tiles_rows(int(R), int(e_local), int(tile_rows)))


def tile_rows_for(records: int, e_local: int, hidden: int, intermediate: int) -> int:
    """Tile height ``moe_layer_forward`` would pick for this many routing
    records over ``e_local`` experts: 256 (CTA-pair GEMMs) once the average
    expert has enough rows, else 128."""
    return int(_native.load().moe_layer_tile_rows(int(records), int(hidden), int(intermediate),
                                                  int(e_local), 1))


def sort_align(ids: torch.Tensor, num_experts: int, e_begin: int = 0, e_local: int | None = None,
               want_inv: bool = False, want_offsets64: bool = False,
               tile_rows: int = 128) -> SortResult:
    """Stable sort of the flat routing records by expert plus the tile table of
    ``tile_rows``-row blocks (C5/python/solution.py:131-136,
    C6/python/solution.py:141-160, C9/python/solution.py:142-159)."""
    _need(ids, "ids", torch.int32)
    flat = ids.reshape(-1)
    R = flat.numel()
    e_local = num_experts if e_local is None else e_local
    dev = ids.device
    lib = _native.load()
    mt = int(lib.moe_max_tiles_rows(R, e_local, tile_rows))
    if mt <= 0 and R >= 0:
        raise ValueError(f"tile_rows must be 128 or 256, got {tile_rows}")
    ws_bytes = int(lib.moe_sort_align_workspace_bytes(R, e_local))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    counts = torch.empty(e_local, dtype=torch.int32, device=dev)
    offsets = torch.empty(e_local + 1, dtype=torch.int32, device=dev)
    off64 = torch.empty(e_local + 1, dtype=torch.int64, device=dev) if want_offsets64 else None
    perm = torch.empty(max(R, 1), dtype=torch.int32, device=dev)[:R]
    inv = torch.empty(R, dtype=torch.int32, device=dev) if want_inv else None
    tiles = torch.empty((max(mt, 1), 4), dtype=torch.int32, device=dev)
    num_tiles = torch.empty(1, dtype=torch.int32, device=dev)
    _rc(lib.moe_sort_align_rows(_p(flat), R, num_experts, e_begin, e_local, _p(ws), ws_bytes,
                                _p(counts), _p(offsets), _p(off64), _p(perm), _p(inv), _p(tiles),
                                mt, _p(num_tiles), tile_rows, _p(status_word(dev)), _stream(dev)),
        "moe_sort_align_rows")
    return SortResult(counts, offsets, off64, perm, inv, tiles, num_tiles, mt, tile_rows)


def tiles_from_offsets(offsets: torch.Tensor, M: int):
    """128-row tile table from int64 offsets[E+1] (C9/python/solution.py:142-159)."""
    _need(offsets, "offsets", torch.int64, 1)
    E = offsets.numel() - 1
    dev = offsets.device
    lib = _native.load()
    mt = int(lib.moe_max_tiles(M, E))
    tiles = torch.empty((max(mt, 1), 4), dtype=torch.int32, device=dev)
    num_tiles = torch.empty(1, dtype=torch.int32, device=dev)
    _rc(lib.moe_tiles_from_offsets(_p(offsets), E, _p(tiles), mt, _p(num_tiles),
                                   _p(status_word(dev)), _stream(dev)), "moe_tiles_from_offsets")
    return tiles, num_tiles, mt


# --------------------------------------------------------------------------- rows


def gather_rows(src: torch.Tensor, index: torch.Tensor, index_div: int = 1,
                count: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """dst[p] = src[index[p] // index_div] (C5/python/solution.py:135-137)."""
    _need(src, "src", torch.bfloat16, 2)
    _need(index, "index", torch.int32, 1)
    R = index.numel()
    H = src.shape[1]
    dst = out if out is not None else torch.empty((R, H), dtype=src.dtype, device=src.device)
    if count is not None:
        _need(count, "count", torch.int32)
    lib = _native.load()
    _rc(lib.moe_gather_rows(_p(src), src.shape[0], _p(index), R, _p(count), index_div, H, _p(dst),
                            _p(status_word(src.device)), _stream(src.device)), "moe_gather_rows")
    return dst


def combine(rows: torch.Tensor, T: int, k: int, slot_src: torch.Tensor | None = None,
            slot_w: torch.Tensor | None = None, ids: torch.Tensor | None = None,
            e_range: tuple[int, int] | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """y[n] = sum_j w_j * rows[src_j] (C5/python/solution.py:158-160)."""
    _need(rows, "rows", torch.bfloat16, 2)
    H = rows.shape[1]
    dev = rows.device
    for name, t, dt in (("slot_src", slot_src, torch.int32), ("slot_w", slot_w, torch.float32),
                        ("ids", ids, torch.int32)):
        if t is not None:
            _need(t, name, dt)
            if t.numel() != T * k:
                raise ValueError(f"{name} must hold T*k = {T * k} entries")
    e0, e1 = e_range if e_range is not None else (0, 1 << 30)
    y = out if out is not None else torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    lib = _native.load()
    _rc(lib.moe_combine(_p(rows), rows.shape[0], _p(slot_src), _p(slot_w), _p(ids), e0, e1, T, k,
                        H, _p(y), _p(status_word(dev)), _stream(dev)), "moe_combine")
    return y


# --------------------------------------------------------------------------- grouped GEMMs


def grouped_w13_swiglu(a: torch.Tensor, tiles: torch.Tensor, num_tiles: torch.Tensor,
                       max_tiles_: int, w_gate: torch.Tensor, w_up: torch.Tensor,
                       out: torch.Tensor | None = None, tile_rows: int = 128) -> torch.Tensor:
    """h = silu(a @ w_gate[e]^T) * (a @ w_up[e]^T) per tile (C9/python/solution.py:218-220)."""
    _need(a, "a", torch.bfloat16, 2)
    _need(w_gate, "w_gate", torch.bfloat16, 3)
    _need(w_up, "w_up", torch.bfloat16, 3)
    M, H = a.shape
    E, I, H2 = w_gate.shape
    if H2 != H or tuple(w_up.shape) != (E, I, H):
        raise ValueError("w_gate / w_up must be [E, I, H] matching a [M, H]")
    h = out if out is not None else torch.empty((M, I), dtype=torch.bfloat16, device=a.device)
    lib = _native.load()
    _rc(lib.moe_grouped_w13_swiglu_rows(_p(a), M, _p(tiles), _p(num_tiles), max_tiles_,
                                        _p(w_gate), _p(w_up), E, H, I, _p(h), tile_rows,
                                        _p(status_word(a.device)), _stream(a.device)),
        "moe_grouped_w13_swiglu_rows")
    return h


def grouped_w13_swiglu_gather(src: torch.Tensor, index: torch.Tensor, index_div: int, M: int,
                              tiles: torch.Tensor, num_tiles: torch.Tensor, max_tiles_: int,
                              w_gate: torch.Tensor, w_up: torch.Tensor,
                              out: torch.Tensor | None = None, tile_rows: int = 128,
                              max_sms: int = 0) -> torch.Tensor:
    """``grouped_w13_swiglu`` whose A row r is ``src[index[r] // index_div]``: the
    permutation gather (C5/python/solution.py:137) fused into the GEMM.
    ``max_sms`` > 0 caps the SMs the GEMM occupies (others stay free for
    concurrent work); the result does not depend on it."""
    _need(src, "src", torch.bfloat16, 2)
    _need(index, "index", torch.int32)
    _need(w_gate, "w_gate", torch.bfloat16, 3)
    _need(w_up, "w_up", torch.bfloat16, 3)
    H = src.shape[1]
    E, I, H2 = w_gate.shape
    if H2 != H or tuple(w_up.shape) != (E, I, H):
        raise ValueError("w_gate / w_up must be [E, I, H] matching src [S, H]")
    if index.numel() < M:
        raise ValueError("index must hold at least M entries")
    h = out if out is not None else torch.empty((M, I), dtype=torch.bfloat16, device=src.device)
    lib = _native.load()
    _rc(lib.moe_grouped_w13_swiglu_gather_ex(_p(src), src.shape[0], _p(index), index_div, M,
                                             _p(tiles), _p(num_tiles), max_tiles_, _p(w_gate),
                                             _p(w_up), E, H, I, _p(h), tile_rows, int(max_sms),
                                             _p(status_word(src.device)), _stream(src.device)),
        "moe_grouped_w13_swiglu_gather_ex")
    return h


def grouped_w2(h: torch.Tensor, tiles: torch.Tensor, num_tiles: torch.Tensor, max_tiles_: int,
               w_down: torch.Tensor, row_map: torch.Tensor | None = None,
               slot_scale: torch.Tensor | None = None, out: torch.Tensor | None = None,
               out_rows: int | None = None, tile_rows: int = 128,
               max_sms: int = 0) -> torch.Tensor:
    """out[map(r)] = scale(map(r)) * (h[r] @ w_down[e]^T) (C9/python/solution.py:221);
    ``max_sms`` as for ``grouped_w13_swiglu_gather``."""
    _need(h, "h", torch.bfloat16, 2)
    _need(w_down, "w_down", torch.bfloat16, 3)
    M, I = h.shape
    E, H, I2 = w_down.shape
    if I2 != I:
        raise ValueError("w_down must be [E, H, I] matching h [M, I]")
    if row_map is not None:
        _need(row_map, "row_map", torch.int32)
    if slot_scale is not None:
        _need(slot_scale, "slot_scale", torch.float32)
    if out is None:
        out = torch.empty((out_rows if out_rows is not None else M, H), dtype=torch.bfloat16,
                          device=h.device)
    lib = _native.load()
    _rc(lib.moe_grouped_w2_ex(_p(h), M, _p(tiles), _p(num_tiles), max_tiles_, _p(w_down), E, H,
                              I, _p(row_map), _p(slot_scale), _p(out), out.shape[0], tile_rows,
                              int(max_sms), _p(status_word(h.device)), _stream(h.device)),
        "moe_grouped_w2_ex")
    return out


INDEX_ADD_MODES = {"deterministic": 0, "atomic": 1}  # MOE_COMBINE_SLOTS / MOE_COMBINE_ATOMIC


def _combine_mode(index_add: str) -> int:
    if index_add not in INDEX_ADD_MODES:
        raise ValueError(f"index_add must be one of {tuple(INDEX_ADD_MODES)}, got {index_add!r}")
    return INDEX_ADD_MODES[index_add]


def grouped_w2_atomic(h: torch.Tensor, tiles: torch.Tensor, num_tiles: torch.Tensor,
                      max_tiles_: int, w_down: torch.Tensor, row_map: torch.Tensor | None,
                      slot_scale: torch.Tensor | None, n_slots: int, red_div: int,
                      out_f32: torch.Tensor, tile_rows: int = 128) -> torch.Tensor:
    """out_f32[map(r) // red_div] += scale(map(r)) * (h[r] @ w_down[e]^T) with fp32
    atomics: the index_add_ un-permute of C5/python/solution.py:158-160 fused into
    the down GEMM.  ``out_f32`` [n_slots // red_div, H] must start at zero."""
    _need(h, "h", torch.bfloat16, 2)
    _need(w_down, "w_down", torch.bfloat16, 3)
    _need(out_f32, "out_f32", torch.float32, 2)
    M, I = h.shape
    E, H, I2 = w_down.shape
    if I2 != I or out_f32.shape[1] != H or out_f32.shape[0] * red_div < n_slots:
        raise ValueError("w_down must be [E, H, I] matching h [M, I]; out_f32 [n_slots/red_div, H]")
    if row_map is not None:
        _need(row_map, "row_map", torch.int32)
    if slot_scale is not None:
        _need(slot_scale, "slot_scale", torch.float32)
    _rc(_native.load().moe_grouped_w2_atomic_rows(
        _p(h), M, _p(tiles), _p(num_tiles), max_tiles_, _p(w_down), E, H, I, _p(row_map),
        _p(slot_scale), n_slots, red_div, _p(out_f32), tile_rows, _p(status_word(h.device)),
        _stream(h.device)), "moe_grouped_w2_atomic_rows")
    return out_f32


def cast_f32_bf16(src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 copy of an fp32 tensor (element count a multiple of 8)."""
    _need(src, "src", torch.float32)
    y = out if out is not None else torch.empty(src.shape, dtype=torch.bfloat16, device=src.device)
    _rc(_native.load().moe_cast_f32_to_bf16(_p(src), src.numel(), _p(y), _stream(src.device)),
        "moe_cast_f32_to_bf16")
    return y


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
                delta: torch.Tensor | None = None):
    """RMSNorm of the rows of ``x`` (or of ``h = x + delta`` in bf16), as the
    decoder block around C8's MoE computes it (C8/python/solution.py:235-325):
    fp32 ``h * rsqrt(mean(h^2) + eps) * weight`` rounded to bf16.  Returns
    ``y`` or ``(h, y)`` when ``delta`` is given."""
    _need(x, "x", torch.bfloat16)
    H = x.shape[-1]
    T = x.numel() // max(H, 1)
    if delta is not None:
        _need(delta, "delta", torch.bfloat16)
        if delta.shape != x.shape:
            raise ValueError("delta must have the shape of x")
    w = weight.detach().float().contiguous()
    if w.device != x.device or w.numel() != H:
        raise ValueError("weight must be [H] on the device of x")
    y = torch.empty_like(x)
    h = torch.empty_like(x) if delta is not None else None
    _rc(_native.load().moe_add_rmsnorm(_p(x), _p(delta), _p(w), T, H, float(eps), _p(h), _p(y),
                                       _stream(x.device)), "moe_add_rmsnorm")
    return (h, y) if delta is not None else y


# --------------------------------------------------------------------------- EP send plan


def ep_keys(ids: torch.Tensor, experts_per_rank: int, ep: int) -> torch.Tensor:
    """keys[n, r] = r if one of token n's experts lives on rank r, else ep
    (the send plan of the one-row-per-owner all_to_all dispatch)."""
    _need(ids, "ids", torch.int32, 2)
    N, k = ids.shape
    keys = torch.empty((N, ep), dtype=torch.int32, device=ids.device)
    _rc(_native.load().moe_ep_keys(_p(ids), N, k, experts_per_rank, ep, _p(keys),
                                   _p(status_word(ids.device)), _stream(ids.device)), "moe_ep_keys")
    return keys


def ep_meta(perm: torch.Tensor, count: torch.Tensor, max_rows: int, ids: torch.Tensor,
            w: torch.Tensor, experts_per_rank: int, ep: int) -> torch.Tensor:
    """Per send row i (pair perm[i] = n*ep + r): int32 [2k] row of token n's
    local expert ids on rank r (experts_per_rank where not on r) and the
    matching weights bit-cast (0 where not on r)."""
    _need(perm, "perm", torch.int32)
    _need(count, "count", torch.int32)
    _need(ids, "ids", torch.int32, 2)
    _need(w, "w", torch.float32, 2)
    N, k = ids.shape
    meta = torch.empty((max_rows, 2 * k), dtype=torch.int32, device=ids.device)
    _rc(_native.load().moe_ep_meta(_p(perm), _p(count), max_rows, _p(ids), _p(w), N, k,
                                   experts_per_rank, ep, _p(meta), _p(status_word(ids.device)),
                                   _stream(ids.device)), "moe_ep_meta")
    return meta


# --------------------------------------------------------------------------- whole layer


def moe_layer(x: torch.Tensor, router_weight: torch.Tensor, w_gate: torch.Tensor,
              w_up: torch.Tensor, w_down: torch.Tensor, top_k: int, norm_topk_prob: bool = True,
              bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None,
              index_add: str = "deterministic",
              w_down_t: torch.Tensor | None = None) -> torch.Tensor:
    """Single-device MoE layer (C5/python/solution.py:108-161) in one C-ABI call.
    ``index_add``: "deterministic" (slot rows + k-sum in slot order, bitwise
    reproducible) or "atomic" (fp32 atomic accumulation per token, the
    reference's index_add_ on CUDA; decode-size batches keep the slot rows).
    ``w_down_t`` (optional, [E, I, H]): with it, batches of up to 4 tokens and
    32 records take the one-pass decode layer (``decode_layer_split``)."""
    mode = _combine_mode(index_add)
    if (w_down_t is not None and mode == 0 and x.dim() == 2 and 0 < x.shape[0] <= 4
            and x.shape[0] * top_k <= 32 and x.shape[1] <= 2048):
        try:
            return decode_layer_split(x, router_weight, w_gate, w_up, w_down_t, top_k,
                                      norm_topk_prob, bias, out, workspace)
        except MoEKernelError as err:
            if err.code != RC_UNSUPPORTED:
                raise
    _need(x, "x", torch.bfloat16, 2)
    for name, t in (("router_weight", router_weight), ("w_gate", w_gate), ("w_up", w_up),
                    ("w_down", w_down)):
        _need(t, name, torch.bfloat16)
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    T, H = x.shape
    E, I, _ = w_gate.shape
    lib = _native.load()
    ws_bytes = int(lib.moe_layer_workspace_bytes_ex(T, H, I, E, top_k, mode))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    y = out if out is not None else torch.empty_like(x)
    if mode == 0:
        _rc(lib.moe_layer_forward(_p(x), _p(router_weight), _p(bias), _p(w_gate), _p(w_up),
                                  _p(w_down), T, H, I, E, top_k, int(bool(norm_topk_prob)),
                                  _p(workspace), workspace.numel(), _p(y),
                                  _p(status_word(x.device)), _stream(x.device)),
            "moe_layer_forward")
    else:
        _rc(lib.moe_layer_forward_ex(_p(x), _p(router_weight), _p(bias), _p(w_gate), _p(w_up),
                                     _p(w_down), T, H, I, E, top_k, int(bool(norm_topk_prob)),
                                     mode, _p(workspace), workspace.numel(), _p(y),
                                     _p(status_word(x.device)), _stream(x.device)),
            "moe_layer_forward_ex")
    return y


def transpose_down_weights(w_down: torch.Tensor) -> torch.Tensor:
    """w_down [E, H, I] -> w_down_t [E, I, H], the layout of the one-pass
    decode layer (built once next to the weights)."""
    _need(w_down, "w_down", torch.bfloat16, 3)
    return w_down.transpose(1, 2).contiguous()


def decode_layer_workspace_bytes(T: int, H: int, E: int) -> int:
    """Workspace bytes of ``decode_layer_split``."""
    return int(_native.load().moe_decode_layer_workspace_bytes(T, H, E))


def decode_layer_split(x: torch.Tensor, router_weight: torch.Tensor, w_gate: torch.Tensor,
                       w_up: torch.Tensor, w_down_t: torch.Tensor, top_k: int,
                       norm_topk_prob: bool = True, bias: torch.Tensor | None = None,
                       out: torch.Tensor | None = None,
                       workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The decode layer (T <= 4, T * top_k <= 32) in one launch and one pass
    over the weights, on transposed down weights ``w_down_t`` [E, I, H].
    Raises if it cannot run (no fallback); equals ``moe_layer`` up to fp32
    summation order."""
    _need(x, "x", torch.bfloat16, 2)
    for name, t in (("router_weight", router_weight), ("w_gate", w_gate), ("w_up", w_up),
                    ("w_down_t", w_down_t)):
        _need(t, name, torch.bfloat16)
    if bias is not None:
        _need(bias, "bias", torch.float32, 1)
    T, H = x.shape
    E, I, _ = w_gate.shape
    if tuple(w_down_t.shape) != (E, I, H):
        raise ValueError(f"w_down_t must be [E, I, H] = {(E, I, H)}, got {tuple(w_down_t.shape)}")
    lib = _native.load()
    ws_bytes = int(lib.moe_decode_layer_workspace_bytes(T, H, E))
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    y = out if out is not None else torch.empty_like(x)
    rc = lib.moe_decode_layer_split(_p(x), _p(router_weight), _p(bias), _p(w_gate), _p(w_up),
                                    _p(w_down_t), T, H, I, E, top_k, int(bool(norm_topk_prob)),
                                    _p(workspace), workspace.numel(), _p(y),
                                    _p(status_word(x.device)), _stream(x.device))
    if rc != 0:
        raise MoEKernelError(f"moe_decode_layer_split: {_native.error_string(rc)} (rc={rc}, "
                             f"cuda error {lib.moe_last_cuda_error()})", rc)
    return y


def device_sm_count() -> int:
    """SMs of the current CUDA device."""
    return int(_native.load().moe_device_sm_count())


def layer_workspace_bytes(T: int, H: int, I: int, E: int, top_k: int,
                          index_add: str = "deterministic") -> int:
    return int(_native.load().moe_layer_workspace_bytes_ex(T, H, I, E, top_k,
                                                           _combine_mode(index_add)))
