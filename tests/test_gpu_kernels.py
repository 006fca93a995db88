"""Parity of each CUDA kernel (through the C ABI) with the CPU oracle.

Integer outputs (ids, counts, offsets, permutation, tile table) must be
bit-exact; floating-point outputs must satisfy the tolerances written in
each test.
"""

import numpy as np
import pytest
import torch

from helpers import to_f32
from moe_inference_verify_microbench_b200 import ops
from oracle import moe_oracle as mo

pytestmark = pytest.mark.gpu


# ----------------------------------------------------------------------------- sort / align


@pytest.mark.parametrize("R,E,e_begin,e_local", [
    (1, 16, 0, 16), (37, 16, 0, 16), (4095, 128, 0, 128), (4096, 128, 0, 128),
    (4097, 128, 0, 128), (40000, 128, 0, 128), (20000, 128, 32, 16), (9000, 64, 48, 16),
])
def test_sort_align_bit_exact(cuda, R, E, e_begin, e_local):
    rng = np.random.default_rng(R + E)
    ids = rng.integers(0, E, size=R).astype(np.int32)
    ids[rng.random(R) < 0.3] = rng.integers(0, max(1, E // 8))  # skew + empty experts
    res = ops.sort_align(torch.from_numpy(ids).to(cuda), E, e_begin, e_local, want_inv=True,
                         want_offsets64=True)
    ops.check_status(cuda)
    loc = ids.astype(np.int64) - e_begin
    keep = (loc >= 0) & (loc < e_local)
    order = np.argsort(np.where(keep, loc, e_local), kind="stable")
    n_keep = int(keep.sum())
    perm_ref = order[:n_keep]
    counts_ref = np.bincount(loc[keep], minlength=e_local)
    offs_ref = np.concatenate([[0], np.cumsum(counts_ref)])
    assert np.array_equal(res.counts.cpu().numpy(), counts_ref)
    assert np.array_equal(res.offsets.cpu().numpy(), offs_ref)
    assert np.array_equal(res.offsets64.cpu().numpy(), offs_ref)
    assert np.array_equal(res.perm[:n_keep].cpu().numpy(), perm_ref)
    inv_ref = np.full(R, -1, dtype=np.int64)
    inv_ref[perm_ref] = np.arange(n_keep)
    assert np.array_equal(res.inv.cpu().numpy(), inv_ref)
    te, tie = mo.tile_metadata(offs_ref, ops.BLOCK_M)
    nt = int(res.num_tiles.item())
    assert nt == len(te)
    tiles = res.tiles[:nt].cpu().numpy()
    assert np.array_equal(tiles[:, 0], te)
    rb = offs_ref[te] + tie * ops.BLOCK_M
    assert np.array_equal(tiles[:, 1], rb)
    assert np.array_equal(tiles[:, 2], np.minimum(offs_ref[te + 1], rb + ops.BLOCK_M))


def test_sort_align_flags_bad_expert(cuda):
    ids = torch.tensor([0, 3, 99, 1], dtype=torch.int32, device=cuda)
    ops.sort_align(ids, 16)
    with pytest.raises(ops.MoEKernelError, match="expert id out of range"):
        ops.check_status(cuda)


def test_tiles_from_offsets(cuda):
    counts = np.array([5, 0, 128, 129, 0, 300, 1], dtype=np.int64)
    offs = np.concatenate([[0], np.cumsum(counts)])
    tiles, nt, mt = ops.tiles_from_offsets(torch.from_numpy(offs).to(cuda), int(offs[-1]))
    te, tie = mo.tile_metadata(offs, ops.BLOCK_M)
    n = int(nt.item())
    assert n == len(te) <= mt
    t = tiles[:n].cpu().numpy()
    assert np.array_equal(t[:, 0], te)
    assert np.array_equal(t[:, 1], offs[te] + tie * ops.BLOCK_M)


# ----------------------------------------------------------------------------- rows


def test_gather_rows_bit_exact(cuda):
    rng = np.random.default_rng(3)
    T, k, H = 300, 8, 256
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    perm = rng.permutation(T * k).astype(np.int32)
    out = ops.gather_rows(x.to(cuda), torch.from_numpy(perm).to(cuda), k)
    ops.check_status(cuda)
    assert torch.equal(out.cpu(), x[torch.from_numpy(perm // k).long()])


def test_gather_rows_device_count(cuda):
    x = torch.arange(40 * 8, dtype=torch.float32).reshape(40, 8).to(torch.bfloat16).to(cuda)
    idx = torch.arange(39, -1, -1, dtype=torch.int32, device=cuda)
    cnt = torch.tensor([7], dtype=torch.int32, device=cuda)
    out = torch.zeros(40, 8, dtype=torch.bfloat16, device=cuda)
    ops.gather_rows(x, idx, 1, count=cnt, out=out)
    ops.check_status(cuda)
    assert torch.equal(out[:7], x.flip(0)[:7])
    assert torch.count_nonzero(out[7:]) == 0


def test_combine_weighted_indirect(cuda):
    g = torch.Generator().manual_seed(1)
    T, k, H = 97, 8, 512
    rows = torch.randn(T * k, H, generator=g).to(torch.bfloat16)
    src = torch.randperm(T * k, generator=g).to(torch.int32)
    w = torch.rand(T * k, generator=g)
    ids = torch.randint(0, 16, (T * k,), generator=g, dtype=torch.int32)
    y = ops.combine(rows.to(cuda), T, k, slot_src=src.to(cuda), slot_w=w.to(cuda),
                    ids=ids.to(cuda), e_range=(4, 12))
    ops.check_status(cuda)
    keep = ((ids >= 4) & (ids < 12)).float()
    ref = (rows.float()[src.long()] * (w * keep)[:, None]).reshape(T, k, H).sum(1)
    assert (y.float().cpu() - ref).abs().max() <= 1e-2 * ref.abs().max()


# ----------------------------------------------------------------------------- router


@pytest.mark.parametrize("T,H,E,k,norm,bias", [
    (1, 256, 16, 4, True, False), (5, 256, 128, 8, True, False), (128, 512, 128, 8, True, True),
    (300, 2048, 128, 8, True, False), (257, 256, 64, 8, False, False), (1000, 2048, 128, 8, False, True),
    (20000, 256, 128, 8, True, False), (4096, 2048, 128, 8, True, True),
])
def test_router_topk(cuda, T, H, E, k, norm, bias):
    """Router logits, top-k ids and weights against the oracle.  Up to 16
    tokens: the cluster kernel on the CUDA cores; up to 8 tiles of 128 tokens:
    the K-split cluster kernel (router_splitk, 2 to 8 ranks per tile); more
    (T=4096, 20000 here): one tcgen05 CTA per tile."""
    d = mo.make_inputs(T, H, 64, E, seed=T, experts=False)
    x = mo.f32_from_bf16_bits(d["x"])
    wr = mo.f32_from_bf16_bits(d["wr"])
    b = mo.zipf_bias(E) if bias else None
    xt = torch.from_numpy(x).to(torch.bfloat16).to(cuda)
    wt = torch.from_numpy(wr).to(torch.bfloat16).to(cuda)
    bt = torch.from_numpy(b).to(cuda) if bias else None
    ids, w, logits = ops.router_topk(xt, wt, k, norm, bias=bt, return_logits=True)
    ops.check_status(cuda)
    lg = to_f32(logits)
    # Logits: fp32 accumulation in another order may move the bf16 rounding by an
    # ulp (more, relatively, for logits that nearly cancel to zero).
    ref_lg = mo.router_logits(x, wr, b)
    assert np.mean(lg != ref_lg) < 0.02
    assert np.all(np.abs(lg - ref_lg) <= np.maximum(np.abs(ref_lg) * 2 ** -7, 1e-3))
    # Routing on the kernel's own logits: ids bit-exact, weights to fp32 rounding.
    vals, ref_ids = mo.topk_ids(lg, k)
    assert np.array_equal(ids.cpu().numpy(), ref_ids)
    ref_w = mo.topk_weights(lg, vals, ref_ids, norm, mode="fp32")
    np.testing.assert_allclose(w.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)


def test_router_tie_rule(cuda):
    """Equal logits: larger value first, then the lower expert id (stable sort order)."""
    T, H, E, k = 4, 64, 32, 8
    x = torch.zeros(T, H)
    x[:, 0] = 1.0
    wr = torch.zeros(E, H)
    wr[:, 0] = torch.tensor([float(v) for v in [1, 2, 2, 0, 2, 3, 3, 1] * 4])
    ids, w, _ = ops.router_topk(x.to(torch.bfloat16).to(cuda), wr.to(torch.bfloat16).to(cuda), k)
    ops.check_status(cuda)
    exp = torch.sort(wr[:, 0], descending=True, stable=True).indices[:k].to(torch.int32)
    assert torch.equal(ids.cpu(), exp.expand(T, k))


# ----------------------------------------------------------------------------- grouped GEMMs


def _grouped_setup(cuda, counts, H, I, seed):
    rng = np.random.default_rng(seed)
    E = len(counts)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    M = int(offs[-1])
    a = (rng.standard_normal((M, H), dtype=np.float32)).astype(np.float32)
    wg = rng.standard_normal((E, I, H), dtype=np.float32) * 0.05
    wu = rng.standard_normal((E, I, H), dtype=np.float32) * 0.05
    wd = rng.standard_normal((E, H, I), dtype=np.float32) * 0.05
    bf = lambda v: torch.from_numpy(v).to(torch.bfloat16)  # noqa: E731
    tb = {k: bf(v) for k, v in dict(a=a, wg=wg, wu=wu, wd=wd).items()}
    fb = {k: v.float().numpy() for k, v in tb.items()}
    tiles, nt, mt = ops.tiles_from_offsets(torch.from_numpy(offs).to(cuda), M)
    return offs, M, tb, fb, tiles, nt, mt


@pytest.mark.parametrize("counts,H,I", [
    ([1, 0, 127, 128, 129, 300, 0, 5], 256, 128),   # BN=256 path
    ([64, 0, 200, 1], 128, 64),                     # BN=128 path
    ([513, 1024, 0, 3], 2048, 768),                 # production shapes
])
def test_w13_swiglu(cuda, counts, H, I):
    offs, M, tb, fb, tiles, nt, mt = _grouped_setup(cuda, counts, H, I, sum(counts))
    h = ops.grouped_w13_swiglu(tb["a"].to(cuda), tiles, nt, mt, tb["wg"].to(cuda), tb["wu"].to(cuda))
    ops.check_status(cuda)
    ref = np.zeros((M, I), dtype=np.float32)
    for e in range(len(counts)):
        s, t = offs[e], offs[e + 1]
        if s == t:
            continue
        g = fb["a"][s:t] @ fb["wg"][e].T
        u = fb["a"][s:t] @ fb["wu"][e].T
        ref[s:t] = mo.silu_f32(g) * u
    assert mo.rel_err(to_f32(h), ref) <= 1e-2


@pytest.mark.parametrize("counts,H,I,mapped", [
    ([1, 0, 127, 128, 129, 300, 0, 5], 256, 128, False),
    ([1, 0, 127, 128, 129, 300, 0, 5], 256, 128, True),
    ([64, 0, 200, 1], 128, 64, True),
    ([513, 1024, 0, 3], 2048, 768, True),
])
def test_w2_scatter(cuda, counts, H, I, mapped):
    offs, M, tb, fb, tiles, nt, mt = _grouped_setup(cuda, counts, H, I, 7 + sum(counts))
    rng = np.random.default_rng(1)
    h = torch.from_numpy(rng.standard_normal((M, I), dtype=np.float32)).to(torch.bfloat16)
    hf = h.float().numpy()
    rmap = rng.permutation(M).astype(np.int32) if mapped else np.arange(M, dtype=np.int32)
    scale = rng.random(M).astype(np.float32) if mapped else np.ones(M, dtype=np.float32)
    out = ops.grouped_w2(h.to(cuda), tiles, nt, mt, tb["wd"].to(cuda),
                         row_map=torch.from_numpy(rmap).to(cuda) if mapped else None,
                         slot_scale=torch.from_numpy(scale).to(cuda) if mapped else None)
    ops.check_status(cuda)
    ref = np.zeros((M, H), dtype=np.float32)
    for e in range(len(counts)):
        s, t = offs[e], offs[e + 1]
        if s < t:
            ref[rmap[s:t]] = (hf[s:t] @ fb["wd"][e].T) * scale[rmap[s:t]][:, None]
    assert mo.rel_err(to_f32(out), ref) <= 1e-2


def _pair_table(offs, cuda):
    """256-row tile table of the CTA-pair GEMMs: every expert's rows cut into
    blocks of 256; a last block of <= 128 rows is a half tile."""
    t = []
    for e in range(len(offs) - 1):
        for b in range(int(offs[e]), int(offs[e + 1]), 256):
            t.append((e, b, min(b + 256, int(offs[e + 1])), 0))
    tiles = torch.tensor(t, dtype=torch.int32, device=cuda).reshape(-1, 4)
    n = torch.tensor([len(t)], dtype=torch.int32, device=cuda)
    return tiles, n, len(t)


@pytest.mark.parametrize("counts,H,I", [
    # half tiles of 1, 64, 65, 127 and 128 rows (M = 128 MMAs) next to full ones
    ([1, 64, 65, 127, 128, 129, 0, 200, 256, 257, 383, 384, 385, 513], 256, 128),
    ([1050, 1000, 1024, 1088, 64, 0, 130], 2048, 768),  # production widths
])
def test_pair_gemms_half_and_full_tiles(cuda, counts, H, I):
    """CTA-pair GEMMs on 256-row tile tables whose last block of an expert may
    hold <= 128 rows (then the pair runs M = 128 MMAs, 64 rows per CTA, with
    the accumulator split over the lane halves): gate/up + SwiGLU with the A
    rows by TMA and gathered by the loader warps (bitwise equal), and the down
    GEMM with the weighted scatter and with the atomic combine, against fp32."""
    offs, M, tb, fb, _, _, _ = _grouped_setup(cuda, counts, H, I, 31 + sum(counts))
    tiles, nt, mt = _pair_table(offs, cuda)
    a = tb["a"].to(cuda)
    wg, wu, wd = (tb[n].to(cuda) for n in ("wg", "wu", "wd"))
    h = ops.grouped_w13_swiglu(a, tiles, nt, mt, wg, wu, tile_rows=256)
    idx = torch.arange(M, dtype=torch.int32, device=cuda)
    h2 = ops.grouped_w13_swiglu_gather(a, idx, 1, M, tiles, nt, mt, wg, wu, tile_rows=256)
    rng = np.random.default_rng(5)
    rmap = rng.permutation(M).astype(np.int32)
    scale = rng.random(M).astype(np.float32)
    rmap_t, scale_t = torch.from_numpy(rmap).to(cuda), torch.from_numpy(scale).to(cuda)
    out = ops.grouped_w2(h, tiles, nt, mt, wd, row_map=rmap_t, slot_scale=scale_t, tile_rows=256)
    acc = torch.zeros(M, H, dtype=torch.float32, device=cuda)
    ops.grouped_w2_atomic(h, tiles, nt, mt, wd, rmap_t, scale_t, M, 1, acc, tile_rows=256)
    ops.check_status(cuda)
    assert torch.equal(h, h2)
    href = np.zeros((M, I), dtype=np.float32)
    oref = np.zeros((M, H), dtype=np.float32)
    hf = to_f32(h)
    for e in range(len(counts)):
        s, t = offs[e], offs[e + 1]
        if s == t:
            continue
        g = fb["a"][s:t] @ fb["wg"][e].T
        u = fb["a"][s:t] @ fb["wu"][e].T
        href[s:t] = mo.silu_f32(g) * u
        oref[rmap[s:t]] = (hf[s:t] @ fb["wd"][e].T) * scale[rmap[s:t]][:, None]
    assert mo.rel_err(hf, href) <= 1e-2
    assert mo.rel_err(to_f32(out), oref) <= 1e-2
    assert mo.rel_err(acc.cpu().numpy(), oref) <= 1e-2


@pytest.mark.parametrize("T,rows", [(2048, 128), (16384, 256), (4, 128)])
def test_sm_budget_leaves_results_bitwise_equal(cuda, T, rows):
    """The grouped GEMMs (and the decode GEMVs, T=4) on at most 16 SMs
    (moe_grouped_*_ex with max_sms) produce bit for bit what they produce on
    every SM: the budget only changes how work units are spread."""
    H, I, E, k = 2048, 768, 128, 8
    g = torch.Generator(device=cuda)
    g.manual_seed(T + rows)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=cuda).to(bf)
    wr = (torch.randn(E, H, generator=g, device=cuda) * 0.02).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.02).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.02).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=cuda) * 0.02).to(bf)
    ids, w, _ = ops.router_topk(x, wr, k)
    s = ops.sort_align(ids, E, tile_rows=rows)
    outs = []
    for budget in (0, 16):
        h = ops.grouped_w13_swiglu_gather(x, s.perm, k, T * k, s.tiles, s.num_tiles, s.max_tiles,
                                          wg, wu, tile_rows=rows, max_sms=budget)
        sl = ops.grouped_w2(h, s.tiles, s.num_tiles, s.max_tiles, wd, row_map=s.perm,
                            slot_scale=w.reshape(-1), tile_rows=rows, max_sms=budget)
        outs.append((h, sl))
    ops.check_status(cuda)
    assert ops.device_sm_count() > 16
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("T,k,H,I,E", [(300, 8, 256, 128, 16), (77, 4, 128, 64, 8), (2048, 8, 2048, 768, 128)])
def test_w13_gather_fused_equals_gather_then_gemm(cuda, T, k, H, I, E):
    """The fused-gather A operand (cp.async, swizzled by hand) must reproduce the
    TMA-loaded pre-gathered operand bit for bit."""
    g = torch.Generator(device=cuda)
    g.manual_seed(T)
    x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
    ids = torch.randint(0, E, (T, k), generator=g, device=cuda, dtype=torch.int32)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(torch.bfloat16)
    s = ops.sort_align(ids, E)
    xs = ops.gather_rows(x, s.perm, k)
    h_ref = ops.grouped_w13_swiglu(xs, s.tiles, s.num_tiles, s.max_tiles, wg, wu)
    h = ops.grouped_w13_swiglu_gather(x, s.perm, k, T * k, s.tiles, s.num_tiles, s.max_tiles, wg, wu)
    ops.check_status(cuda)
    assert torch.equal(h, h_ref)


def test_layer_uses_fused_gather_consistently(cuda):
    """moe_layer_forward (fused gather) equals the op-by-op pipeline with the
    explicit gather, bit for bit."""
    T, H, I, E, k = 700, 256, 128, 16, 4
    g = torch.Generator(device=cuda)
    g.manual_seed(1)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=cuda).to(bf)
    wr = (torch.randn(E, H, generator=g, device=cuda) * 0.05).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=cuda) * 0.05).to(bf)
    y = ops.moe_layer(x, wr, wg, wu, wd, k)
    ids, w, _ = ops.router_topk(x, wr, k)
    s = ops.sort_align(ids, E)
    xs = ops.gather_rows(x, s.perm, k)
    h = ops.grouped_w13_swiglu(xs, s.tiles, s.num_tiles, s.max_tiles, wg, wu)
    sl = ops.grouped_w2(h, s.tiles, s.num_tiles, s.max_tiles, wd, row_map=s.perm,
                        slot_scale=w.reshape(-1))
    y2 = ops.combine(sl, T, k)
    ops.check_status(cuda)
    assert torch.equal(y, y2)


# ----------------------------------------------------------------------------- decode (GEMV) path


@pytest.mark.parametrize("counts,H,I", [
    ([1, 0, 3, 8, 0, 2, 1, 1], 2048, 768),        # decode shapes, a few records per expert
    ([20, 1, 0, 9, 2], 256, 128),                 # > 8 records per expert: several passes
    ([128], 512, 64),                             # largest gate/up batch on the streaming path
])
def test_gemv_w13_w2_small_batches(cuda, counts, H, I):
    """Small batches run the expert GEMMs as weight-streaming GEMVs (gate/up up
    to 128 records, down up to 32); same contract (tile table, row map, slot
    scale, fused gather) as the tensor-core kernels."""
    offs, M, tb, fb, tiles, nt, mt = _grouped_setup(cuda, counts, H, I, 3 + sum(counts))
    assert M <= 128
    h = ops.grouped_w13_swiglu(tb["a"].to(cuda), tiles, nt, mt, tb["wg"].to(cuda), tb["wu"].to(cuda))
    # Fused gather through an index with a divisor: A row p = src[index[p] // 2].
    src = torch.zeros(2 * M, H, dtype=torch.bfloat16)
    perm = torch.randperm(M, generator=torch.Generator().manual_seed(M)).to(torch.int32)
    src[perm.long()] = tb["a"]
    index = 2 * perm + torch.arange(M, dtype=torch.int32) % 2
    h_g = ops.grouped_w13_swiglu_gather(src.to(cuda), index.to(cuda), 2, M, tiles, nt, mt,
                                        tb["wg"].to(cuda), tb["wu"].to(cuda))
    rng = np.random.default_rng(5)
    rmap = rng.permutation(M).astype(np.int32)
    scale = rng.random(M).astype(np.float32)
    out = ops.grouped_w2(h, tiles, nt, mt, tb["wd"].to(cuda), row_map=torch.from_numpy(rmap).to(cuda),
                         slot_scale=torch.from_numpy(scale).to(cuda))
    ops.check_status(cuda)
    assert torch.equal(h_g, h)
    hf = to_f32(h)
    ref_h = np.zeros((M, I), dtype=np.float32)
    ref_o = np.zeros((M, H), dtype=np.float32)
    for e in range(len(counts)):
        s, t = offs[e], offs[e + 1]
        if s == t:
            continue
        g = fb["a"][s:t] @ fb["wg"][e].T
        u = fb["a"][s:t] @ fb["wu"][e].T
        ref_h[s:t] = mo.silu_f32(g) * u
        ref_o[rmap[s:t]] = (hf[s:t] @ fb["wd"][e].T) * scale[rmap[s:t]][:, None]
    assert mo.rel_err(hf, ref_h) <= 1e-2
    assert mo.rel_err(to_f32(out), ref_o) <= 1e-2


def _decode_reference_f32(x, wr, wg, wu, wd, ids, w, k):
    """fp32 torch restatement of the layer for given routing: bf16 h as the
    kernels round it, fp32 down projection, bf16 slot rows, fp32 k-sum."""
    T = x.shape[0]
    xf = x.float()
    y = torch.zeros(T, x.shape[1], device=x.device)
    for n in range(T):
        for j in range(k):
            e = int(ids[n, j])
            h = (torch.nn.functional.silu(xf[n] @ wg[e].float().T) * (xf[n] @ wu[e].float().T))
            h = h.to(torch.bfloat16).float()
            y[n] += ((wd[e].float() @ h) * w[n, j]).to(torch.bfloat16).float()
    return y


@pytest.mark.parametrize("T,norm,with_bias", [(1, True, False), (2, False, False), (4, True, True),
                                              (6, True, False), (8, False, True)])
def test_single_launch_decode_layer_bitwise(cuda, T, norm, with_bias):
    """Up to 64 routing records (T <= 8 at top-8) run the whole layer as one
    cooperative launch (router, top-k, sort, both GEMVs and the combine, with
    grid barriers between them).  Its output must equal the four-launch
    decode pipeline, op by op through the C ABI, bit for bit, at the full
    shapes (H=2048 I=768 E=128 k=8)."""
    H, I, E, k = 2048, 768, 128, 8
    g = torch.Generator(device=cuda)
    g.manual_seed(500 + T)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=cuda).to(bf)
    wr = (torch.randn(E, H, generator=g, device=cuda) * 0.02).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.02).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.02).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=cuda) * 0.02).to(bf)
    bias = torch.randn(E, generator=g, device=cuda) * 0.1 if with_bias else None
    y = ops.moe_layer(x, wr, wg, wu, wd, k, norm_topk_prob=norm, bias=bias)
    y_again = ops.moe_layer(x, wr, wg, wu, wd, k, norm_topk_prob=norm, bias=bias)
    ids, w, _ = ops.router_topk(x, wr, k, norm_topk_prob=norm, bias=bias)
    s = ops.sort_align(ids, E)
    h = ops.grouped_w13_swiglu_gather(x, s.perm, k, T * k, s.tiles, s.num_tiles, s.max_tiles,
                                      wg, wu)
    sl = ops.grouped_w2(h, s.tiles, s.num_tiles, s.max_tiles, wd, row_map=s.perm,
                        slot_scale=w.reshape(-1))
    y2 = ops.combine(sl, T, k)
    ops.check_status(cuda)
    assert torch.equal(y, y2)
    assert torch.equal(y, y_again)


def _decode_reference_f32(x, wr, wg, wu, wd, ids, w, k):
    """fp32 torch restatement of the layer for given routing: bf16 h as the
    kernels round it, fp32 down projection, bf16 slot rows, fp32 k-sum."""
    T = x.shape[0]
    xf = x.float()
    y = torch.zeros(T, x.shape[1], device=x.device)
    for n in range(T):
        for j in range(k):
            e = int(ids[n, j])
            h = (torch.nn.functional.silu(xf[n] @ wg[e].float().T) * (xf[n] @ wu[e].float().T))
            h = h.to(torch.bfloat16).float()
            y[n] += ((wd[e].float() @ h) * w[n, j]).to(torch.bfloat16).float()
    return y


@pytest.mark.parametrize("T,norm,with_bias", [(1, True, False), (2, False, False), (3, True, False),
                                              (4, True, True)])
def test_one_pass_decode_layer(cuda, T, norm, with_bias):
    """The one-pass decode layer on transposed down weights (router, top-k,
    sort, one split-I stream over gate, up and w_down_t, segment sums and the
    combine, one launch) at the full shapes (H=2048 I=768 E=128 k=8): equal
    to the layer's own decode path up to fp32 summation order (at least 98 %
    of the elements bit for bit, the rest within the bf16 rounding of the slot
    rows), within 1e-2 of an fp32 restatement, and repeatable bit for bit.
    ``moe_layer`` given w_down_t runs the same kernel."""
    H, I, E, k = 2048, 768, 128, 8
    g = torch.Generator(device=cuda)
    g.manual_seed(500 + T)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=cuda).to(bf)
    wr = (torch.randn(E, H, generator=g, device=cuda) * 0.02).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.02).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.02).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=cuda) * 0.02).to(bf)
    wdt = ops.transpose_down_weights(wd)
    bias = torch.randn(E, generator=g, device=cuda) * 0.1 if with_bias else None
    y = ops.decode_layer_split(x, wr, wg, wu, wdt, k, norm_topk_prob=norm, bias=bias)
    y_again = ops.decode_layer_split(x, wr, wg, wu, wdt, k, norm_topk_prob=norm, bias=bias)
    y_layer = ops.moe_layer(x, wr, wg, wu, wd, k, norm_topk_prob=norm, bias=bias, w_down_t=wdt)
    y2 = ops.moe_layer(x, wr, wg, wu, wd, k, norm_topk_prob=norm, bias=bias)
    ids, w, _ = ops.router_topk(x, wr, k, norm_topk_prob=norm, bias=bias)
    ops.check_status(cuda)
    assert torch.equal(y, y_again) and torch.equal(y, y_layer)
    assert (y == y2).float().mean().item() >= 0.98
    d = (y.float() - y2.float()).abs()
    assert d.max().item() <= 2.0 ** -7 * y2.float().abs().max().item()
    yref = _decode_reference_f32(x, wr, wg, wu, wd, ids, w, k)
    assert ((y.float() - yref).norm() / yref.norm()).item() <= 1e-2


@pytest.mark.parametrize("T,k,E,I", [(1, 4, 16, 128), (1, 8, 16, 16), (4, 8, 64, 128),
                                     (2, 1, 128, 768)])
def test_one_pass_decode_layer_ragged_ranges(cuda, T, k, E, I):
    """Small shapes where most CTAs get an empty item range, a tile spans a
    single item or two (I=16), or one CTA range covers several tiles: the
    segment bookkeeping of the one-pass decode layer must still sum every
    partial once."""
    H = 256
    g = torch.Generator(device=cuda)
    g.manual_seed(900 + T * 10 + I)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=cuda).to(bf)
    wr = (torch.randn(E, H, generator=g, device=cuda) * 0.05).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=cuda) * 0.05).to(bf)
    y = ops.decode_layer_split(x, wr, wg, wu, ops.transpose_down_weights(wd), k)
    ids, w, _ = ops.router_topk(x, wr, k)
    ops.check_status(cuda)
    yref = _decode_reference_f32(x, wr, wg, wu, wd, ids, w, k)
    assert ((y.float() - yref).norm() / yref.norm()).item() <= 1e-2


@pytest.mark.parametrize("T,k,E", [(1, 4, 16), (3, 8, 64), (16, 8, 128), (17, 4, 32)])
def test_layer_decode_equals_op_by_op(cuda, T, k, E):
    """moe_layer_forward at decode sizes (fused router + sort, GEMV experts)
    equals the op-by-op pipeline through the separate C-ABI entry points, bit
    for bit."""
    H, I = 256, 128
    g = torch.Generator(device=cuda)
    g.manual_seed(T * 100 + E)
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g, device=cuda).to(bf)
    wr = (torch.randn(E, H, generator=g, device=cuda) * 0.05).to(bf)
    wg = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(bf)
    wu = (torch.randn(E, I, H, generator=g, device=cuda) * 0.05).to(bf)
    wd = (torch.randn(E, H, I, generator=g, device=cuda) * 0.05).to(bf)
    y = ops.moe_layer(x, wr, wg, wu, wd, k)
    ids, w, _ = ops.router_topk(x, wr, k)
    s = ops.sort_align(ids, E)
    xs = ops.gather_rows(x, s.perm, k)
    h = ops.grouped_w13_swiglu(xs, s.tiles, s.num_tiles, s.max_tiles, wg, wu)
    sl = ops.grouped_w2(h, s.tiles, s.num_tiles, s.max_tiles, wd, row_map=s.perm,
                        slot_scale=w.reshape(-1))
    y2 = ops.combine(sl, T, k)
    ops.check_status(cuda)
    assert torch.equal(y, y2)


# ----------------------------------------------------------------------------- EP send plan


@pytest.mark.parametrize("N,k,E,ep", [(1000, 8, 128, 2), (4096, 8, 128, 8), (77, 4, 16, 4)])
def test_ep_plan_kernels_match_torch(cuda, N, k, E, ep):
    """moe_ep_keys / moe_ep_meta equal their torch formulation, bit for bit."""
    g = torch.Generator(device=cuda)
    g.manual_seed(N + ep)
    scores = torch.rand(N, E, generator=g, device=cuda)
    ids = scores.topk(k, dim=1).indices.to(torch.int32)      # distinct experts per token
    w = torch.softmax(torch.rand(N, k, generator=g, device=cuda), dim=1)
    epr = E // ep
    keys = ops.ep_keys(ids, epr, ep)
    dest = ids.long() // epr
    sent = torch.zeros((N, ep), dtype=torch.bool, device=cuda)
    sent.scatter_(1, dest, True)
    ranks = torch.arange(ep, dtype=torch.int32, device=cuda)
    assert torch.equal(keys, torch.where(sent, ranks, torch.full_like(ranks, ep)))
    plan = ops.sort_align(keys, ep + 1, 0, ep, want_inv=True)
    total = int(plan.offsets[ep].item())
    meta = ops.ep_meta(plan.perm, plan.offsets[ep:], total, ids, w, epr, ep)
    ops.check_status(cuda)
    pair = plan.perm[:total].long()
    tok, rank_of = pair // ep, pair % ep
    own = dest.index_select(0, tok) == rank_of[:, None]
    meta_e = torch.where(own, ids.index_select(0, tok) - (rank_of * epr)[:, None].to(torch.int32),
                         torch.full_like(ids[:1], epr)).to(torch.int32)
    meta_w = (w.index_select(0, tok) * own).contiguous().view(torch.int32)
    assert torch.equal(meta, torch.cat([meta_e, meta_w], dim=1))


# ----------------------------------------------------------------------------- block glue


@pytest.mark.parametrize("T,H", [(1, 2048), (37, 2048), (4096, 2048), (5, 64)])
def test_add_rmsnorm_matches_harness(cuda, T, H):
    """moe_add_rmsnorm against the harness RMSNorm (fp32 math, bf16 out); the
    residual sum is bf16 addition, bit-exact."""
    from moe_inference_verify_microbench_b200.hybrid import RMSNorm
    g = torch.Generator(device=cuda)
    g.manual_seed(T + H)
    x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
    a = (torch.randn(T, H, generator=g, device=cuda) * 0.5).to(torch.bfloat16)
    norm = RMSNorm(H, eps=1e-6).to(cuda)
    norm.weight.data.copy_(1.0 + 0.1 * torch.randn(H, generator=g, device=cuda))
    y1 = ops.add_rmsnorm(x, norm.weight, norm.eps)
    h, y2 = ops.add_rmsnorm(x, norm.weight, norm.eps, delta=a)
    with torch.no_grad():
        r1 = norm(x)
        hr = x + a
        r2 = norm(hr)
    assert torch.equal(h, hr)
    assert mo.rel_err(to_f32(y1), to_f32(r1)) <= 1e-2
    assert mo.rel_err(to_f32(y2), to_f32(r2)) <= 1e-2
    # most elements agree to the bit; the rest differ by one bf16 step
    assert (y2 == r2).float().mean().item() >= 0.95
