"""A torch-CPU stand-in for the kernel contract of ``ep.CudaKernels``.

Test infrastructure only: it lets the expert-parallel schedules' host logic
(split sizes, collective order, index bookkeeping) run on gloo ranks without
a GPU.  It follows the same index conventions as the CUDA kernels (stable
sort, slot = n*k + j, inv = -1 outside the expert range)."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from moe_inference_verify_microbench_b200.ops import SortResult


class CpuContractKernels:
    @staticmethod
    def router_topk(x, wr, k, norm_topk_prob=True, bias=None, return_logits=False):
        acc = x.float() @ wr.float().T
        if bias is not None:
            acc = acc + bias.float()
        logits = acc.to(torch.bfloat16).float()
        ids = torch.sort(logits, dim=-1, descending=True, stable=True).indices[:, :k]
        if norm_topk_prob:
            w = torch.softmax(torch.gather(logits, 1, ids), dim=-1)
        else:
            w = torch.gather(torch.softmax(logits, dim=-1), 1, ids)
        return ids.to(torch.int32), w.float(), logits.to(torch.bfloat16)

    @staticmethod
    def tile_rows(expected_records, e_local, hidden, intermediate):
        return 128

    @staticmethod
    def sort_align(ids, num_experts, e_begin=0, e_local=None, want_inv=False, want_offsets64=False,
                   tile_rows=128):
        e_local = num_experts if e_local is None else e_local
        flat = ids.reshape(-1).long()
        loc = flat - e_begin
        keep = (loc >= 0) & (loc < e_local)
        key = torch.where(keep, loc, torch.full_like(loc, e_local))
        order = torch.sort(key, stable=True).indices
        n = int(keep.sum())
        counts = torch.bincount(loc[keep], minlength=e_local)
        offsets = F.pad(counts.cumsum(0), (1, 0))
        perm = torch.zeros(flat.numel(), dtype=torch.int32)
        perm[:n] = order[:n].to(torch.int32)
        inv = torch.full((flat.numel(),), -1, dtype=torch.int32)
        inv[order[:n]] = torch.arange(n, dtype=torch.int32)
        return SortResult(counts.to(torch.int32), offsets.to(torch.int32), offsets, perm, inv,
                          None, torch.tensor([0]), 0)

    @staticmethod
    def ep_keys(ids, epr, ep):
        dest = ids.long() // epr
        sent = torch.zeros((ids.shape[0], ep), dtype=torch.bool)
        sent.scatter_(1, dest, True)
        ranks = torch.arange(ep, dtype=torch.int32)
        return torch.where(sent, ranks, torch.full_like(ranks, ep))

    @staticmethod
    def ep_meta(perm, count, max_rows, ids, w, epr, ep):
        pair = perm[:max_rows].long()
        tok = pair // ep
        rank_of = pair - tok * ep
        own = ids.index_select(0, tok).long() // epr == rank_of[:, None]
        meta_e = torch.where(own, ids.index_select(0, tok) - (rank_of * epr)[:, None].to(torch.int32),
                             torch.full_like(ids[:1], epr)).to(torch.int32)
        meta_w = w.index_select(0, tok) * own
        return torch.cat([meta_e, meta_w.contiguous().view(torch.int32)], dim=1)

    @staticmethod
    def gather_rows(src, index, index_div=1, count=None, out=None):
        n = index.numel() if count is None else min(index.numel(), int(count.reshape(-1)[0]))
        dst = torch.zeros((index.numel(), src.shape[1]), dtype=src.dtype)
        dst[:n] = src[index[:n].long() // index_div]
        return dst

    @staticmethod
    def expert_compute(src, index, index_div, s, w_gate, w_up, w_down, row_map=None,
                       slot_scale=None, out_rows=None, max_sms=0):
        M = index.numel()
        n = int(s.offsets[-1])
        xs = torch.zeros((M, src.shape[1]), dtype=src.dtype)
        xs[:n] = src[index[:n].long() // index_div]
        out = torch.zeros((out_rows if out_rows is not None else M, w_down.shape[1]),
                          dtype=torch.bfloat16)
        off = s.offsets.tolist()
        for e in range(len(off) - 1):
            a, b = off[e], off[e + 1]
            if a == b:
                continue
            xe = xs[a:b].float()
            h = (F.silu(xe @ w_gate[e].float().T) * (xe @ w_up[e].float().T)).to(torch.bfloat16)
            o = h.float() @ w_down[e].float().T
            rows = torch.arange(a, b) if row_map is None else row_map[a:b].long()
            if slot_scale is not None:
                o = o * slot_scale[rows][:, None]
            out[rows] = o.to(torch.bfloat16)
        return out

    @staticmethod
    def combine(rows, T, k, slot_src=None, slot_w=None, ids=None, e_range=None, out=None):
        s = torch.arange(T * k) if slot_src is None else slot_src.reshape(-1).long()
        w = torch.ones(T * k) if slot_w is None else slot_w.reshape(-1).float()
        valid = s >= 0
        if ids is not None and e_range is not None:
            e = ids.reshape(-1).long()
            valid &= (e >= e_range[0]) & (e < e_range[1])
        contrib = rows.float()[s.clamp(min=0)] * (w * valid)[:, None]
        y = contrib.reshape(T, k, rows.shape[1]).sum(1).to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y


class CpuPeerExchange:
    """A torch-CPU model of ``peer.PeerExchange`` on gloo ranks: the buffer
    contents the exchange kernels leave behind (receive rows source-major,
    unfilled receive rows carrying the sentinel expert id, returned rows in
    send order), moved with all_to_all instead of peer stores."""

    def __init__(self, group, cap_rows, hidden, top_k):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.ep = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.cap_rows, self.hidden, self.top_k = cap_rows, hidden, top_k
        self.broken = False
        self.recv_ids = torch.zeros((cap_rows, top_k), dtype=torch.int32)
        self.recv_w = torch.zeros((cap_rows, top_k), dtype=torch.float32)
        self.recv_rows = torch.zeros((cap_rows, hidden), dtype=torch.bfloat16)
        self.ret_rows = torch.zeros((cap_rows, hidden), dtype=torch.bfloat16)

    def _a2a(self, t, send, recv):
        from moe_inference_verify_microbench_b200.dist_primer import all_to_all_variable
        return all_to_all_variable(t, send, recv, self.group)

    def dispatch(self, send_counts, x, perm, ids, weights, experts_per_rank):
        ep, epr = self.ep, experts_per_rank
        counts = send_counts[:ep].to(torch.int64).contiguous()
        recv = torch.empty_like(counts)
        self.dist.all_to_all_single(recv, counts, group=self.group)
        self._send, self._recv = counts.tolist(), recv.tolist()
        total = sum(self._send)
        assert x.shape[0] * ep <= self.cap_rows and sum(self._recv) <= self.cap_rows
        pairs = perm[:total].long()
        n, d = pairs // ep, pairs % ep
        e = ids[n].long()
        own = (e // epr) == d[:, None]
        loc = torch.where(own, e - d[:, None] * epr, torch.full_like(e, epr)).to(torch.int32)
        wt = torch.where(own, weights[n], torch.zeros_like(weights[n]))
        rx = self._a2a(x[n], self._send, self._recv)
        nr = rx.shape[0]
        self._nr = nr
        self.recv_rows[:nr] = rx
        self.recv_ids[:nr] = self._a2a(loc, self._send, self._recv)
        self.recv_ids[nr:] = epr
        self.recv_w[:nr] = self._a2a(wt, self._send, self._recv)

    def give_back(self, out, inv):
        nr, k = self._nr, self.top_k
        slot = inv.reshape(-1)[:nr * k].long().reshape(nr, k)
        valid = slot >= 0
        contrib = out.float()[slot.clamp(min=0)] * (self.recv_w[:nr] * valid)[..., None]
        part = contrib.sum(1).to(torch.bfloat16)
        back = self._a2a(part, self._recv, self._send)
        self.ret_rows[:back.shape[0]] = back

    def close(self):
        pass
