"""One rank's side of the peer-store expert-parallel exchange
(``moe_ep_peer_*`` in include/moe_b200.h).

The all_to_all schedule of C7/python/solution.py:186-261 (and C8's MoE,
C8/python/solution.py:171-224) exchanges split sizes with a count all_to_all,
reads them on the host (``.tolist()``, C7:199-200) and moves rows with three
variable all_to_alls.  Here every rank owns one device buffer that its peers
write into over NVLink (CUDA IPC mappings): the split sizes, the dispatched
rows with their routing metadata, and the returned partial rows, each step
signalled by an epoch flag.  Nothing in a forward synchronises the host, so
the forward can be captured in a CUDA graph.

The buffers are exchanged once, collectively, when the object is built; every
rank of the group must build it at the same point with the same capacity.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native, ops

IPC_HANDLE_BYTES = 64
MAX_RANKS = 8

_REGION_RECV_IDS, _REGION_RECV_W, _REGION_RECV_ROWS, _REGION_RET_ROWS = 0, 1, 2, 3


class _DeviceView:
    """A typed view of device memory this module allocated itself, consumable
    by ``torch.as_tensor`` (CUDA array interface, version 3)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self.__cuda_array_interface__ = {
            "shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
            "strides": None,
        }


def _view(ptr: int, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device):
    typestr = {torch.int32: "<i4", torch.float32: "<f4", torch.bfloat16: "<i2"}[dtype]
    t = torch.as_tensor(_DeviceView(ptr, shape, typestr), device=device)
    return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t


def _all_gather(obj, group):
    if not dist.is_available() or not dist.is_initialized():
        return [obj]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out


class PeerExchange:
    """Peer buffers of an expert-parallel group, mapped into this process.

    ``cap_rows`` bounds both the rows this rank sends (one per (token, owner
    rank) pair: at most ep x tokens) and the rows it receives; pass ep x the
    largest per-rank token count of any forward.  ``group`` None with no
    process group initialised means a group of one rank.
    """

    def __init__(self, group, cap_rows: int, hidden: int, top_k: int,
                 device: torch.device) -> None:
        if dist.is_available() and dist.is_initialized():
            self.ep = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.ep, self.rank = 1, 0
        if self.ep > MAX_RANKS:
            raise ValueError(f"the peer exchange supports at most {MAX_RANKS} ranks, got {self.ep}")
        if hidden % 8 or top_k < 1 or top_k > 8 or cap_rows < 0:
            raise ValueError("peer exchange needs hidden % 8 == 0, 1 <= top_k <= 8, cap_rows >= 0")
        self.cap_rows, self.hidden, self.top_k = int(cap_rows), int(hidden), int(top_k)
        self.device = torch.device(device)
        self.group = group
        # Set by the expert-parallel modules when a forward saw a peer timeout:
        # the ranks' epochs may disagree from then on, so the exchange is not reused.
        self.broken = False
        lib = _native.load()
        self._lib = lib
        nbytes = int(lib.moe_ep_peer_buffer_bytes(self.ep, self.cap_rows, hidden, top_k))
        if nbytes == 0:
            raise ValueError("invalid peer exchange shape")
        own = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            ops._rc(lib.moe_ep_peer_alloc(nbytes, ctypes.byref(own), handle), "moe_ep_peer_alloc")
        self._own = own.value
        self._opened: list[int] = []
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        recs = _all_gather((bytes(handle), uuid, self.cap_rows, hidden, top_k), group)
        try:
            if len({r[1] for r in recs}) != self.ep:
                raise RuntimeError("ranks of the expert-parallel group share a GPU; the peer "
                                   "exchange needs one GPU per rank")
            if any(tuple(r[2:]) != (self.cap_rows, hidden, top_k) for r in recs):
                raise RuntimeError("ranks disagree on the peer exchange shape "
                                   f"{[tuple(r[2:]) for r in recs]}")
            bases = (ctypes.c_void_p * MAX_RANKS)()
            for q, r in enumerate(recs):
                if q == self.rank:
                    bases[q] = self._own
                    continue
                h = (ctypes.c_ubyte * IPC_HANDLE_BYTES).from_buffer_copy(r[0])
                p = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    ops._rc(lib.moe_ep_peer_open(h, ctypes.byref(p)), "moe_ep_peer_open")
                self._opened.append(p.value)
                bases[q] = p.value
        except Exception:
            self._release()
            raise
        self._bases = bases
        off = lambda region: self._own + int(lib.moe_ep_peer_region_offset(  # noqa: E731
            self.ep, self.cap_rows, hidden, top_k, region))
        cap, k, H, dev = self.cap_rows, top_k, hidden, self.device
        self.recv_ids = _view(off(_REGION_RECV_IDS), (cap, k), torch.int32, dev)
        self.recv_w = _view(off(_REGION_RECV_W), (cap, k), torch.float32, dev)
        self.recv_rows = _view(off(_REGION_RECV_ROWS), (cap, H), torch.bfloat16, dev)
        self.ret_rows = _view(off(_REGION_RET_ROWS), (cap, H), torch.bfloat16, dev)

    def dispatch(self, send_counts: torch.Tensor, x: torch.Tensor, perm: torch.Tensor,
                 ids: torch.Tensor, weights: torch.Tensor, experts_per_rank: int) -> None:
        """Send row i (pair perm[i] = n*ep + d, rank-major, send_counts[d] rows
        for rank d) to rank d; afterwards (stream order) this rank's
        ``recv_*`` views hold what it received."""
        ops._need(send_counts, "send_counts", torch.int32)
        ops._need(x, "x", torch.bfloat16, 2)
        ops._need(perm, "perm", torch.int32)
        ops._need(ids, "ids", torch.int32, 2)
        ops._need(weights, "weights", torch.float32, 2)
        N = x.shape[0]
        if send_counts.numel() < self.ep or x.shape[1] != self.hidden:
            raise ValueError("send_counts must hold ep entries and x must be [N, hidden]")
        if tuple(ids.shape) != (N, self.top_k) or tuple(weights.shape) != (N, self.top_k):
            raise ValueError("ids / weights must be [N, top_k]")
        if N * self.ep > self.cap_rows:
            raise ValueError(f"{N} tokens x {self.ep} ranks exceed the exchange capacity "
                             f"{self.cap_rows} rows")
        dev = x.device
        ops._rc(self._lib.moe_ep_peer_dispatch(
            self._bases, self.ep, self.rank, self.cap_rows, self.hidden, self.top_k,
            ops._p(send_counts), ops._p(x), N, ops._p(perm), ops._p(ids), ops._p(weights),
            int(experts_per_rank), ops._p(ops.status_word(dev)), ops._stream(dev)),
            "moe_ep_peer_dispatch")

    def give_back(self, out: torch.Tensor, inv: torch.Tensor) -> None:
        """Per received row, the weighted sum of its records' expert outputs
        (record p at ``out[inv[p]]``) back to its source; afterwards (stream
        order) this rank's ``ret_rows`` hold one partial row per send position."""
        ops._need(out, "out", torch.bfloat16, 2)
        ops._need(inv, "inv", torch.int32)
        if inv.numel() < self.cap_rows * self.top_k or out.shape[1] != self.hidden:
            raise ValueError("inv must cover cap_rows * top_k records and out must be [*, hidden]")
        dev = out.device
        ops._rc(self._lib.moe_ep_peer_return(
            self._bases, self.ep, self.rank, self.cap_rows, self.hidden, self.top_k, ops._p(out),
            out.shape[0], ops._p(inv), ops._p(ops.status_word(dev)), ops._stream(dev)),
            "moe_ep_peer_return")

    def _release(self) -> None:
        for p in self._opened:
            self._lib.moe_ep_peer_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own:
            self._lib.moe_ep_peer_free(ctypes.c_void_p(self._own))
            self._own = 0

    def close(self) -> None:
        """Collective: waits for this device, then for every rank, so no peer
        still writes into a buffer that is unmapped or freed."""
        torch.cuda.synchronize(self.device)
        if self.ep > 1:
            dist.barrier(group=self.group)
        for name in ("recv_ids", "recv_w", "recv_rows", "ret_rows"):
            setattr(self, name, None)
        self._release()


def set_wait_limit_ms(ms: int) -> None:
    """Bound of every wait on a peer rank (default 10 s; ms <= 0 restores it)."""
    _native.load().moe_ep_peer_set_wait_limit_ms(int(ms))
