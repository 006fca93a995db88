"""Peer-store expert-parallel exchange on one GPU (``moe_ep_peer_*``):

* a group of one rank runs the whole C7 forward through the exchange kernels
  (publish, dispatch, return, their waits) and must agree with the
  single-GPU layer, over several forwards (epochs) and under CUDA-graph replay;
* a wait on a peer that never signals (rank 0 of a two-rank layout whose
  rank 1 never runs) ends on its bounded limit with MOE_ERR_PEER_TIMEOUT in the
  status word, and the device stays usable.

The multi-rank exchange runs in tests/test_gpu_ep.py (one process per GPU).
"""

import ctypes

import pytest
import torch

from moe_inference_verify_microbench_b200 import _native, ops, peer
from moe_inference_verify_microbench_b200.ep_pure import EPSparseMoE
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8


def _weights(dev, seed=5):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wg = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wu = (torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wd = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    return g, wr, wg, wu, wd


@pytest.mark.parametrize("T", [1, 300, 4096])
def test_peer_exchange_one_rank_matches_layer(cuda, T):
    g, wr, wg, wu, wd = _weights(cuda)
    with torch.device(cuda):
        mod = EPSparseMoE(H, I, E, K, 1, 0, group=None, transport="peer",
                          max_tokens_per_rank=T).to(torch.bfloat16)
    mod.weight_loader(wr, list(wg), list(wu), list(wd))
    try:
        for step in range(3):  # three epochs through the same buffers
            x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
            with torch.no_grad():
                y = mod(x)
                y_ref = ops.moe_layer(x, wr, wg, wu, wd, K)
            torch.cuda.synchronize()
            ops.check_status(cuda)
            err = mo.rel_err(y.float().cpu().numpy(), y_ref.float().cpu().numpy())
            assert err <= 1e-2, (T, step, err)
    finally:
        mod.close()


def test_peer_exchange_graph_replay(cuda):
    T = 2048
    g, wr, wg, wu, wd = _weights(cuda, seed=9)
    with torch.device(cuda):
        mod = EPSparseMoE(H, I, E, K, 1, 0, group=None, transport="peer",
                          max_tokens_per_rank=T).to(torch.bfloat16)
    mod.weight_loader(wr, list(wg), list(wu), list(wd))
    try:
        x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
        with torch.no_grad():
            y_eager = mod(x).clone()
            s = torch.cuda.Stream(cuda)
            s.wait_stream(torch.cuda.current_stream(cuda))
            with torch.cuda.stream(s):
                mod(x)  # warm-up on the capture stream
            torch.cuda.current_stream(cuda).wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                y_graph = mod(x)
            outs = []
            for _ in range(3):
                graph.replay()
                outs.append(y_graph.clone())
        torch.cuda.synchronize()
        ops.check_status(cuda)
        for o in outs:  # the epoch advances on the device at every replay
            assert torch.equal(o, y_eager)
        del graph
    finally:
        mod.close()


def test_peer_wait_times_out_with_status(cuda):
    lib = _native.load()
    ep, cap, k = 2, 64, K
    nbytes = int(lib.moe_ep_peer_buffer_bytes(ep, cap, H, k))
    bufs = []
    handle = (ctypes.c_ubyte * peer.IPC_HANDLE_BYTES)()
    for _ in range(ep):  # both "ranks" on this GPU; rank 1 never runs
        p = ctypes.c_void_p()
        ops._rc(lib.moe_ep_peer_alloc(nbytes, ctypes.byref(p), handle), "moe_ep_peer_alloc")
        bufs.append(p.value)
    bases = (ctypes.c_void_p * peer.MAX_RANKS)(*bufs)
    x = torch.randn(16, H, device=cuda).to(torch.bfloat16)
    ids = torch.randint(0, E, (16, k), device=cuda, dtype=torch.int32)
    w = torch.rand(16, k, device=cuda)
    counts = torch.tensor([16, 16], dtype=torch.int32, device=cuda)
    n = torch.arange(16, dtype=torch.int32, device=cuda)
    perm = torch.cat([n * ep, n * ep + 1])  # rank-major send order of (token, rank) pairs
    st = ops.status_word(cuda)
    st.zero_()
    try:
        peer.set_wait_limit_ms(200)
        rc = lib.moe_ep_peer_dispatch(bases, ep, 0, cap, H, k, ops._p(counts), ops._p(x), 16,
                                      ops._p(perm), ops._p(ids), ops._p(w), E // ep, ops._p(st),
                                      ops._stream(cuda))
        assert rc == 0
        torch.cuda.synchronize()
        assert int(st.item()) == 0x105
        st.zero_()
        # the context is intact: a kernel afterwards runs and reports nothing
        ops.gather_rows(x, torch.arange(16, dtype=torch.int32, device=cuda))
        torch.cuda.synchronize()
        ops.check_status(cuda)
    finally:
        peer.set_wait_limit_ms(0)
        st.zero_()
        for p in bufs:
            lib.moe_ep_peer_free(ctypes.c_void_p(p))
