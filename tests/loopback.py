"""Every rank of an expert-parallel group as a thread of one process on one GPU.

Test infrastructure only.  The schedules in ``ep.py`` call
``torch.distributed`` for their collectives; inside ``LoopbackWorld.run`` those
calls are served by an in-process stand-in, so a single GPU runs the real
CUDA kernels of every rank while the collectives become device copies:

* every rank is a thread; all of them launch on the device's legacy default
  stream, so work runs in the order it was enqueued across threads;
* a collective is a rendezvous of the group's threads (a barrier): each rank
  posts its input, then enqueues its reads of the other ranks' inputs, then
  waits on the barrier a second time before any rank goes on to enqueue work
  that could overwrite those inputs.  Stream order then guarantees that every
  read runs after the kernels that produced its data and before any later
  write to it;
* ``all_reduce`` sums in fp32 in rank order and rounds once (NCCL's bf16
  reduction order is its own; the tests compare within the bf16 tolerance).

Only host-synchronised transports can run this way: kernels that wait on one
another (the peer-store exchange) never run as separate launches on one GPU.
"""

from __future__ import annotations

import threading
from contextlib import contextmanager
from unittest import mock

import torch
import torch.distributed as dist


class _Group:
    def __init__(self, ranks, timeout):
        self.ranks = list(ranks)
        self.barrier = threading.Barrier(len(self.ranks), timeout=timeout)
        self.slots = [None] * len(self.ranks)


class LoopbackWorld:
    def __init__(self, world: int, device: torch.device, timeout: float = 120.0) -> None:
        self.world = world
        self.device = device
        self.timeout = timeout
        self.default = _Group(range(world), timeout)
        self._groups: dict[tuple, _Group] = {}
        self._lock = threading.Lock()
        self._tls = threading.local()

    # ------------------------------------------------------------ helpers
    def _rank(self) -> int:
        return self._tls.rank

    def _g(self, group) -> _Group:
        return self.default if group is None else group

    def _post(self, group, value):
        g = self._g(group)
        i = g.ranks.index(self._rank())
        g.slots[i] = value
        g.barrier.wait()
        return g, i, list(g.slots)

    @staticmethod
    def _release(g: _Group) -> None:
        g.barrier.wait()

    # ------------------------------------------------------------ collectives
    def all_reduce(self, t, op=None, group=None, async_op=False):
        g, _, vals = self._post(group, t)
        acc = vals[0].float()
        for v in vals[1:]:
            acc = acc + v.float()
        self._release(g)
        t.copy_(acc.to(t.dtype))

    def all_to_all_single(self, output, input, output_split_sizes=None, input_split_sizes=None,
                          group=None, async_op=False):
        g, i, vals = self._post(group, (input, input_split_sizes))
        n = len(g.ranks)
        off = 0
        for src, splits in vals:
            sp = [int(s) for s in splits] if splits is not None else [src.shape[0] // n] * n
            start, cnt = sum(sp[:i]), sp[i]
            if cnt:
                output[off:off + cnt].copy_(src[start:start + cnt])
            off += cnt
        self._release(g)

    def all_gather_into_tensor(self, output_tensor, input_tensor, group=None, async_op=False):
        g, _, vals = self._post(group, input_tensor)
        n = input_tensor.shape[0]
        for s, v in enumerate(vals):
            output_tensor[s * n:(s + 1) * n].copy_(v)
        self._release(g)

    def barrier(self, group=None, **kw):
        self._g(group).barrier.wait()

    def new_group(self, ranks=None, **kw):
        key = tuple(range(self.world)) if ranks is None else tuple(ranks)
        with self._lock:
            if key not in self._groups:
                self._groups[key] = _Group(key, self.timeout)
            return self._groups[key]

    def get_world_size(self, group=None):
        return len(self._g(group).ranks)

    def get_rank(self, group=None):
        return self._g(group).ranks.index(self._rank())

    # ------------------------------------------------------------ driver
    @contextmanager
    def _patched(self):
        with mock.patch.multiple(
                dist, all_reduce=self.all_reduce, all_to_all_single=self.all_to_all_single,
                all_gather_into_tensor=self.all_gather_into_tensor, barrier=self.barrier,
                new_group=self.new_group, get_world_size=self.get_world_size,
                get_rank=self.get_rank, is_initialized=lambda: True):
            yield

    def run(self, fn):
        """fn(rank) on every rank's thread; returns the per-rank results.  A
        failure on one rank breaks every barrier, so the others end too, and
        the first failure is raised."""
        results = [None] * self.world
        errors: list[tuple[int, BaseException]] = []

        def body(r):
            self._tls.rank = r
            if self.device.type == "cuda":
                torch.cuda.set_device(self.device)
            try:
                results[r] = fn(r)
            except BaseException as e:  # noqa: BLE001 - reported below
                errors.append((r, e))
                for g in [self.default, *self._groups.values()]:
                    g.barrier.abort()

        with self._patched():
            threads = [threading.Thread(target=body, args=(r,)) for r in range(self.world)]
            for t in threads:
                t.start()
            for t in threads:
                t.join()
        if errors:
            errors.sort(key=lambda e: isinstance(e[1], threading.BrokenBarrierError))
            r, e = errors[0]
            raise RuntimeError(f"rank {r} failed: {e!r}") from e
        return results
