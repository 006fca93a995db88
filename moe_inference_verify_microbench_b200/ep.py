"""Expert-parallel MoE schedules over NCCL, with the call signatures of the
reference's components:

* ``EPSparseMoELean``  C6/python/solution.py:57-182 (exported by ``ep_lean`` as
  ``EPSparseMoE``): replicated input, full router on every rank, local experts
  only, ONE all_reduce of the [N, H] partial output.
* ``EPSparseMoEPure``  C7/python/solution.py:65-269 (exported by ``ep_pure`` as
  ``EPSparseMoE``): distinct tokens per rank; count all_to_all, dispatch
  all_to_all of rows and expert ids, local grouped compute, combine
  all_to_all, weighted k-way combine.
* ``HybridMoE``        C8/python/solution.py:59-230: 1/tp stripe of the
  TP-replicated input, the C7 core on the EP group, all_gather on the TP group.

Experts are sharded contiguously: rank r owns [r*E/ep, (r+1)*E/ep)
(C6:87-89, C7:96-98, C8:110-112).  Every rank issues the same collectives in
the same order as the reference (C8:12-19), so the schedules compose with
the reference's TP attention.  The local compute is the sm_100a kernel set of
``ops``.  With ``transport="nccl"`` (the default) the exchange is NCCL's
variable all_to_all, whose split sizes the host must read (the reference's
``.tolist()``, C7:199-200); with ``transport="peer"`` (C7 and C8) the ranks
write into each other's buffers over NVLink with the split sizes negotiated on
the device (``peer.PeerExchange``): no host synchronisation in the forward.

Errors.  With the keyword extra ``check_errors=True`` every forward
synchronises and raises ``ops.MoEKernelError`` when a kernel reported a
failure in the device status word (an expert id out of range, a peer that did
not signal in time); otherwise failures are only recorded there
(``ops.check_status``).  A peer timeout seen that way marks the exchange
unusable: its ranks' epochs may no longer agree, so later forwards raise
until ``close()`` (collective) and a new forward rebuild it.  A forward whose
batch exceeds the peer capacity (``max_tokens_per_rank``, or the largest
per-rank batch of the first forward) still takes its part in the exchange
step, with an empty batch, so the other ranks' results stay correct and every
rank stays in step, and then raises ``ValueError``.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from . import ops
from .dist_primer import all_to_all_variable
from .experts import ExpertBank, SwiGLU_MLP, router_bias_of
from .peer import PeerExchange, _all_gather

TRANSPORTS = ("nccl", "peer")


class CudaKernels:
    """The kernel contract the schedules are written against (all sm_100a)."""

    router_topk = staticmethod(ops.router_topk)
    sort_align = staticmethod(ops.sort_align)
    ep_keys = staticmethod(ops.ep_keys)
    ep_meta = staticmethod(ops.ep_meta)
    gather_rows = staticmethod(ops.gather_rows)
    combine = staticmethod(ops.combine)

    @staticmethod
    def tile_rows(expected_records, e_local, hidden, intermediate):
        """Tile height for the local grouped GEMMs (256: CTA-pair kernels)."""
        return ops.tile_rows_for(expected_records, e_local, hidden, intermediate)

    @staticmethod
    def expert_compute(src, index, index_div, s, w_gate, w_up, w_down, row_map=None,
                       slot_scale=None, out_rows=None, max_sms=0):
        """SwiGLU experts on rows src[index[p] // index_div] of the sorted order,
        gathered inside the gate/up GEMM (only the rows the tile table covers,
        i.e. the sort's valid records, are read or computed), w2 output to
        row_map[p] scaled by slot_scale[row_map[p]]; both GEMMs on at most
        ``max_sms`` SMs when > 0."""
        M = s.perm.numel()
        h = ops.grouped_w13_swiglu_gather(src, index, index_div, M, s.tiles, s.num_tiles,
                                          s.max_tiles, w_gate, w_up, tile_rows=s.tile_rows,
                                          max_sms=max_sms)
        return ops.grouped_w2(h, s.tiles, s.num_tiles, s.max_tiles, w_down, row_map=row_map,
                              slot_scale=slot_scale, out_rows=out_rows, tile_rows=s.tile_rows,
                              max_sms=max_sms)


class _EPBase(nn.Module):
    def __init__(self, hidden, intermediate, num_experts, top_k, ep_size, ep_rank, norm_topk_prob):
        super().__init__()
        assert num_experts % ep_size == 0, (
            f"num_experts={num_experts} not divisible by ep_size={ep_size}")
        self.hidden = hidden
        self.intermediate = intermediate
        self.num_experts = num_experts
        self.top_k = top_k
        self.ep_size = ep_size
        self.ep_rank = ep_rank
        self.norm_topk_prob = norm_topk_prob
        self.experts_per_rank = num_experts // ep_size
        self.expert_start = ep_rank * self.experts_per_rank
        self.expert_end = self.expert_start + self.experts_per_rank
        # REPLICATED router; SHARDED experts (C6:91-96).
        self.gate = nn.Linear(hidden, num_experts, bias=False)
        self.experts = nn.ModuleList(SwiGLU_MLP(hidden, intermediate)
                                     for _ in range(self.experts_per_rank))
        self._bank = ExpertBank()
        self._kernels = CudaKernels

    def _apply(self, fn, *args, **kwargs):
        self._bank.invalidate()
        return super()._apply(fn, *args, **kwargs)

    def pack(self):
        return self._bank.bind(self.experts)

    @torch.no_grad()
    def weight_loader(self, gate_weight, expert_gate_weights, expert_up_weights,
                      expert_down_weights) -> None:
        """Copy the replicated router and this rank's expert shard
        (C6/python/solution.py:98-110)."""
        self.gate.weight.data.copy_(gate_weight)
        wg, wu, wd = self.pack()
        for local_e in range(self.experts_per_rank):
            global_e = self.expert_start + local_e
            wg[local_e].copy_(expert_gate_weights[global_e])
            wu[local_e].copy_(expert_up_weights[global_e])
            wd[local_e].copy_(expert_down_weights[global_e])

    def _route(self, x_flat):
        return self._kernels.router_topk(x_flat, self.gate.weight, self.top_k, self.norm_topk_prob,
                                         bias=router_bias_of(self.gate))[:2]


class EPSparseMoELean(_EPBase):
    """Replicated-input EP with one all_reduce (C6/python/solution.py:57-182)."""

    def __init__(self, hidden: int, intermediate: int, num_experts: int, top_k: int, ep_size: int,
                 ep_rank: int, group: dist.ProcessGroup | None = None,
                 norm_topk_prob: bool = True, *, check_errors: bool = False) -> None:
        super().__init__(hidden, intermediate, num_experts, top_k, ep_size, ep_rank, norm_topk_prob)
        self.group = group
        self.check_errors = check_errors

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        K = self._kernels
        shape = x.shape
        x_flat = x.reshape(-1, shape[-1]).contiguous()
        N, k = x_flat.shape[0], self.top_k
        ids, w = self._route(x_flat)                                   # full router (C6:127-133)
        rows = K.tile_rows(N * k // self.ep_size, self.experts_per_rank, self.hidden,
                           self.intermediate)                          # expected local records
        s = K.sort_align(ids, self.num_experts, self.expert_start,     # local filter + stable sort
                         self.experts_per_rank, tile_rows=rows)        # (C6:141-160)
        wg, wu, wd = self.pack()
        slots = K.expert_compute(x_flat, s.perm, k, s, wg, wu, wd,     # gather (C6:156) fused;
                                 row_map=s.perm, slot_scale=w.reshape(-1),  # weighted, to slot
                                 out_rows=N * k)                       # rows (C6:163-170)
        partial = K.combine(slots, N, k, ids=ids.reshape(-1),          # (C6:175-176)
                            e_range=(self.expert_start, self.expert_end))
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)  # (C6:180)
        if self.check_errors:
            ops.check_status(partial.device)
        return partial.reshape(shape)


def dispatch_combine(mod: _EPBase, local_x: torch.Tensor, group) -> torch.Tensor:
    """The all_to_all EP core shared by C7 (C7/python/solution.py:120-269) and
    C8's MoE (C8/python/solution.py:171-224), on this rank's tokens.

    The reference dispatches k copies of every token (one per routing record,
    C7:167,201).  Here a token travels once to each rank that owns at least
    one of its experts, with its (local expert, weight) list; the owner runs
    every record of the row through the grouped GEMMs, sums them with their
    weights, and returns one partial row per (token, rank), which the sender
    sums.  Same collectives in the same order (counts, dispatch, combine) and
    the same result; the rows on the wire drop from k per token to the number
    of distinct owner ranks per token.
    """
    K = mod._kernels
    N, k, E, epr, ep = local_x.shape[0], mod.top_k, mod.num_experts, mod.experts_per_rank, mod.ep_size
    ids, w = mod._route(local_x)                                       # local router (C7:141-146)
    # Send plan: key each (token n, rank r) pair with r if one of n's experts lives
    # on r, else the sentinel ep; a stable sort by key gives the per-rank counts,
    # the send order (rank-major, token order inside) and each pair's position.
    keys = K.ep_keys(ids, epr, ep)
    plan = K.sort_align(keys, ep + 1, 0, ep, want_inv=True)
    send = plan.counts.to(torch.int64)                                 # rows per destination
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)                   # count exchange (C7:190)
    send_l, recv_l = send.tolist(), recv.tolist()                     # host sync (C7:199-200)
    total = int(sum(send_l))
    # Per send row (pair n*ep + r): the k local expert ids on r and their
    # weights, one int32 row of 2k entries (weights bit-cast) (C7:203).
    meta = K.ep_meta(plan.perm, plan.offsets[ep:], total, ids, w, epr, ep)
    xs = K.gather_rows(local_x, plan.perm, ep, count=plan.offsets[ep:])[:total]
    recv_x = all_to_all_variable(xs, send_l, recv_l, group)           # dispatch (C7:201)
    recv_m = all_to_all_variable(meta, send_l, recv_l, group)
    recv_e = recv_m[:, :k].contiguous()
    recv_w = recv_m[:, k:].contiguous().view(torch.float32)
    n_recv = recv_x.shape[0]
    wg, wu, wd = mod.pack()
    if n_recv > 0:
        rows = K.tile_rows(n_recv * k // ep, epr, mod.hidden, mod.intermediate)
        s2 = K.sort_align(recv_e, epr + 1, 0, epr, want_inv=True,    # local re-sort (C7:224-226);
                          tile_rows=rows)
        out = K.expert_compute(recv_x, s2.perm, k, s2, wg, wu, wd)    # id epr marks "not mine"
        partial = K.combine(out, n_recv, k, slot_src=s2.inv,          # weighted sum of the row's
                            slot_w=recv_w.reshape(-1))                # records (C7:259-261)
    else:
        partial = recv_x.new_empty((0, local_x.shape[1]))
    back = all_to_all_variable(partial, recv_l, send_l, group)        # combine (C7:258)
    return K.combine(back, N, ep, slot_src=plan.inv)                  # sum over owner ranks (ep <= 8)


def dispatch_combine_peer(mod: _EPBase, local_x: torch.Tensor, px: PeerExchange) -> torch.Tensor:
    """``dispatch_combine`` over the peer-store exchange: the same send plan,
    local compute and combines, with the three all_to_alls and the host read
    of the split sizes replaced by device-signalled stores into the peers'
    buffers.  The receive buffer has a fixed capacity; rows no source filled
    carry the sentinel expert id, so the local sort leaves them out."""
    K = mod._kernels
    N, k, epr, ep = local_x.shape[0], mod.top_k, mod.experts_per_rank, mod.ep_size
    ids, w = mod._route(local_x)                                       # local router (C7:141-146)
    keys = K.ep_keys(ids, epr, ep)
    plan = K.sort_align(keys, ep + 1, 0, ep, want_inv=True)
    px.dispatch(plan.counts, local_x, plan.perm, ids, w, epr)        # counts + dispatch (C7:190-203)
    rows = K.tile_rows(px.cap_rows * k // ep, epr, mod.hidden, mod.intermediate)
    s2 = K.sort_align(px.recv_ids, epr + 1, 0, epr, want_inv=True,  # local re-sort (C7:224-226)
                      tile_rows=rows)
    wg, wu, wd = mod.pack()
    out = K.expert_compute(px.recv_rows, s2.perm, k, s2, wg, wu, wd)
    px.give_back(out, s2.inv)                                          # weighted row sums (C7:258-261)
    return K.combine(px.ret_rows, N, ep, slot_src=plan.inv)           # sum over owner ranks


class _Streams:
    """Side stream and events of the pipelined exchange on a CUDA device; on
    CPU tensors (the gloo stand-ins) every operation runs in program order and
    these are no-ops."""

    def __init__(self, device: torch.device) -> None:
        self.cuda = device.type == "cuda"
        self.side = torch.cuda.Stream(device) if self.cuda else None

    def on_side(self):
        import contextlib
        return torch.cuda.stream(self.side) if self.cuda else contextlib.nullcontext()

    def mark(self, side: bool = False):
        """An event recorded on the side (or the current) stream."""
        if not self.cuda:
            return None
        ev = torch.cuda.Event()
        ev.record(self.side if side else torch.cuda.current_stream())
        return ev

    def side_waits(self, ev) -> None:
        if ev is not None:
            self.side.wait_event(ev)

    def main_waits(self, ev) -> None:
        if ev is not None:
            torch.cuda.current_stream().wait_event(ev)

    def keep(self, *tensors) -> None:
        """Tensors allocated on the main stream and used on the side stream."""
        if self.cuda:
            for t in tensors:
                if t is not None:
                    t.record_stream(self.side)


def dispatch_combine_peer_pipelined(mod: _EPBase, local_x: torch.Tensor, pxs, st: _Streams,
                                    exchange_sms: int) -> torch.Tensor:
    """``dispatch_combine_peer`` in len(pxs) token chunks whose exchanges
    overlap the other chunks' expert GEMMs (D = dispatch, G = local sort and
    GEMMs, R = return of chunk i):

        main stream   D0 | G0       | G1       | ... | G(n-1)   | R(n-1) | combine
        side stream      | D1       | R0, D2   | ... | R(n-2)   |

    The GEMMs leave ``exchange_sms`` SMs free, on which the side stream's
    exchange kernels (SM-issued NVLink stores) run; only the first chunk's
    dispatch and the last chunk's return stay on the critical path, at the
    price of one more pass over the local experts' weights per chunk.  Each
    chunk has its own peer exchange (own buffers and epochs) and every rank
    issues the exchanges in the same order.  A token's records stay in one
    chunk, so every owner rank sums the same records in the same order as in
    the one-chunk forward: the output is bit for bit the same.

    On B200 it measured slower than the one-chunk exchange at 2, 4 and 8
    ranks (16384 tokens per rank): the SM-issued exchange kernels get too few
    SMs beside the persistent GEMMs to hide behind them, and every chunk adds
    a pass over the rank's expert weights.  It is kept as an option."""
    K = mod._kernels
    n_ch = len(pxs)
    N, k, epr, ep = local_x.shape[0], mod.top_k, mod.experts_per_rank, mod.ep_size
    step = -(-N // n_ch)
    bounds = [(min(i * step, N), min((i + 1) * step, N)) for i in range(n_ch)]
    ids, w = mod._route(local_x)                                       # local router (C7:141-146)
    plans = [K.sort_align(K.ep_keys(ids[a:b], epr, ep), ep + 1, 0, ep, want_inv=True)
             for a, b in bounds]
    wg, wu, wd = mod.pack()
    budget = 0
    if st.cuda and exchange_sms > 0:
        budget = max(2, ops.device_sm_count() - int(exchange_sms))
    # Tile height of the one-chunk exchange (a function of the whole batch's
    # capacity), so both forwards run the same GEMM configuration.
    rows = K.tile_rows(n_ch * pxs[0].cap_rows * k // ep, epr, mod.hidden, mod.intermediate)

    def dispatch(i):
        a, b = bounds[i]
        pxs[i].dispatch(plans[i].counts, local_x[a:b], plans[i].perm, ids[a:b], w[a:b], epr)

    dispatch(0)
    if n_ch > 1:
        st.keep(local_x, ids, w, *[t for p in plans[1:] for t in (p.counts, p.perm)])
        st.side_waits(st.mark())               # the plans are ready
        with st.on_side():
            dispatch(1)
    arrived = [None] + [st.mark(side=True) if i == 1 else None for i in range(1, n_ch)]
    for i in range(n_ch):
        st.main_waits(arrived[i])              # chunk i has arrived
        s_i = K.sort_align(pxs[i].recv_ids, epr + 1, 0, epr, want_inv=True, tile_rows=rows)
        out_i = K.expert_compute(pxs[i].recv_rows, s_i.perm, k, s_i, wg, wu, wd,
                                 max_sms=budget if n_ch > 1 else 0)
        if i == n_ch - 1:
            pxs[i].give_back(out_i, s_i.inv)   # the last return: critical path
            break
        st.keep(out_i, s_i.inv)
        st.side_waits(st.mark())               # chunk i's expert outputs are ready
        with st.on_side():
            pxs[i].give_back(out_i, s_i.inv)
            if i + 2 < n_ch:
                dispatch(i + 2)
        if i + 2 < n_ch:
            arrived[i + 2] = st.mark(side=True)
    st.main_waits(st.mark(side=True))          # every return has landed
    y = local_x.new_empty((N, local_x.shape[1]))
    for (a, b), p, px in zip(bounds, plans, pxs):
        K.combine(px.ret_rows, b - a, ep, slot_src=p.inv, out=y[a:b])
    return y


class _A2ABase(_EPBase):
    """Transport selection shared by the all_to_all schedules."""

    def _init_transport(self, transport: str, max_tokens_per_rank: int | None,
                        check_errors: bool, overlap: bool | int = False,
                        exchange_sms: int = 16) -> None:
        if transport not in TRANSPORTS:
            raise ValueError(f"transport must be one of {TRANSPORTS}, got {transport!r}")
        if overlap and transport != "peer":
            raise ValueError("overlap needs transport='peer'")
        chunks = 2 if overlap is True else int(overlap)
        if overlap and chunks < 2:
            raise ValueError(f"overlap takes True or a chunk count >= 2, got {overlap!r}")
        self.transport = transport
        self.max_tokens_per_rank = max_tokens_per_rank
        self.check_errors = check_errors
        self.overlap = bool(overlap)
        self.overlap_chunks = chunks if overlap else 1
        self.exchange_sms = exchange_sms
        self._peer: PeerExchange | None = None
        self._peer_chunks: list | None = None
        self._streams: _Streams | None = None

    def _exchange(self, local_x: torch.Tensor, group) -> torch.Tensor:
        if self.transport == "nccl":
            return dispatch_combine(self, local_x, group)
        if self.overlap:
            return self._exchange_pipelined(local_x, group)
        if self._peer is None:
            # Collective, on the first forward of every rank: the capacity is
            # ep x the largest per-rank token count, then the buffers are swapped.
            n_max = self.max_tokens_per_rank
            if n_max is None:
                n_max = max(_all_gather(local_x.shape[0], group))
            self._peer = PeerExchange(group, self.ep_size * int(n_max), self.hidden, self.top_k,
                                      local_x.device)
        px = self._peer
        if getattr(px, "broken", False):
            raise RuntimeError("the peer exchange timed out in an earlier forward and its ranks "
                               "may be out of step; call close() on every rank to rebuild it")
        if local_x.shape[0] * self.ep_size > px.cap_rows:
            # Refusing before the exchange would leave the peers waiting for this
            # rank's step until they time out, and this rank one epoch behind them
            # for good.  Take part with an empty batch instead, then refuse.
            dispatch_combine_peer(self, local_x[:0], px)
            raise ValueError(f"{local_x.shape[0]} tokens on this rank exceed the peer exchange "
                             f"capacity of {px.cap_rows // self.ep_size} tokens per rank; this "
                             "rank sent nothing in this step (the other ranks' results are "
                             "complete); pass max_tokens_per_rank to size the exchange")
        return dispatch_combine_peer(self, local_x, px)

    def _exchange_pipelined(self, local_x: torch.Tensor, group) -> torch.Tensor:
        n_ch = self.overlap_chunks
        if self._peer_chunks is None:
            # Collective, on the first forward: one exchange per token chunk,
            # each sized for its share of the largest per-rank batch.
            n_max = self.max_tokens_per_rank
            if n_max is None:
                n_max = max(_all_gather(local_x.shape[0], group))
            cap = self.ep_size * (-(-int(n_max) // n_ch))
            self._peer_chunks = [PeerExchange(group, cap, self.hidden, self.top_k, local_x.device)
                                 for _ in range(n_ch)]
            self._streams = _Streams(local_x.device)
        pxs = self._peer_chunks
        if any(getattr(px, "broken", False) for px in pxs):
            raise RuntimeError("the peer exchange timed out in an earlier forward and its ranks "
                               "may be out of step; call close() on every rank to rebuild it")
        if -(-local_x.shape[0] // n_ch) * self.ep_size > pxs[0].cap_rows:
            # As in the one-chunk exchange: take part with an empty batch, then refuse.
            dispatch_combine_peer_pipelined(self, local_x[:0], pxs, self._streams,
                                            self.exchange_sms)
            raise ValueError(f"{local_x.shape[0]} tokens on this rank exceed the peer exchange "
                             f"capacity of {n_ch * pxs[0].cap_rows // self.ep_size} tokens per "
                             "rank; this rank sent nothing in this step; pass "
                             "max_tokens_per_rank to size the exchange")
        return dispatch_combine_peer_pipelined(self, local_x, pxs, self._streams,
                                               self.exchange_sms)

    def _checked(self, y: torch.Tensor) -> torch.Tensor:
        if not self.check_errors:
            return y
        try:
            ops.check_status(y.device)
        except ops.MoEKernelError as err:
            if err.code == ops.ERR_PEER_TIMEOUT:
                for px in [self._peer] + list(self._peer_chunks or []):
                    if px is not None:
                        px.broken = True
            raise
        return y

    def close(self) -> None:
        """Collective with the peer transport: unmap and free the peer buffers."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None
        if self._peer_chunks is not None:
            if self._streams is not None and self._streams.cuda:
                self._streams.side.synchronize()
            for px in self._peer_chunks:
                px.close()
            self._peer_chunks = None


class EPSparseMoEPure(_A2ABase):
    """Pure EP: distinct tokens per rank, dispatch/combine all_to_all
    (C7/python/solution.py:65-269).  The group is kept as ``ep_group`` (C7:93).
    ``transport`` and ``max_tokens_per_rank`` are keyword extras (module
    docstring); the reference's arguments keep their meaning."""

    def __init__(self, hidden: int, intermediate: int, num_experts: int, top_k: int, ep_size: int,
                 ep_rank: int, group: dist.ProcessGroup | None = None,
                 norm_topk_prob: bool = True, *, transport: str = "nccl",
                 max_tokens_per_rank: int | None = None, check_errors: bool = False,
                 overlap: bool | int = False, exchange_sms: int = 16) -> None:
        super().__init__(hidden, intermediate, num_experts, top_k, ep_size, ep_rank, norm_topk_prob)
        self.ep_group = group
        self._init_transport(transport, max_tokens_per_rank, check_errors, overlap, exchange_sms)

    def forward(self, local_x: torch.Tensor) -> torch.Tensor:
        shape = local_x.shape
        x_flat = local_x.reshape(-1, self.hidden).contiguous()
        return self._checked(self._exchange(x_flat, self.ep_group)).reshape(shape)


class HybridMoE(_A2ABase):
    """TP-scoped stripe/all_gather + EP-scoped dispatch/combine
    (C8/python/solution.py:59-230); ``transport`` as for ``EPSparseMoEPure``."""

    def __init__(self, hidden: int, intermediate: int, num_experts: int, top_k: int, tp_size: int,
                 tp_rank: int, tp_group: dist.ProcessGroup | None, ep_size: int, ep_rank: int,
                 ep_group: dist.ProcessGroup | None, norm_topk_prob: bool = True, *,
                 transport: str = "nccl", max_tokens_per_rank: int | None = None,
                 check_errors: bool = False, overlap: bool | int = False,
                 exchange_sms: int = 16) -> None:
        super().__init__(hidden, intermediate, num_experts, top_k, ep_size, ep_rank, norm_topk_prob)
        self.tp_size = tp_size
        self.tp_rank = tp_rank
        self.tp_group = tp_group
        self.ep_group = ep_group
        self._init_transport(transport, max_tokens_per_rank, check_errors, overlap, exchange_sms)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x_flat = x.reshape(-1, self.hidden)
        N_tp = x_flat.shape[0]
        assert N_tp % self.tp_size == 0
        local_N = N_tp // self.tp_size
        local_x = x_flat[self.tp_rank * local_N:(self.tp_rank + 1) * local_N].contiguous()  # (C8:160)
        local_y = self._checked(self._exchange(local_x, self.ep_group))
        y_flat = torch.empty((N_tp, self.hidden), dtype=local_y.dtype, device=local_y.device)
        dist.all_gather_into_tensor(y_flat, local_y, group=self.tp_group)            # (C8:227)
        return y_flat.reshape(shape)
