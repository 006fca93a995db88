"""CPU oracle for the MoE-layer hot path (test infrastructure only).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The CUDA path in
``moe_inference_verify_microbench_b200`` never calls into it.

It restates, in numpy, the reference's single-device MoE algorithm
(weidotwisc/moe_inference_verify_microbench):

* router + top-k + renormalised softmax ........ C5/python/solution.py:124-129
* flatten, argsort by expert, bincount, gather .. C5/python/solution.py:131-138
* per-expert SwiGLU ............................. C5/python/solution.py:68-80, 142-157
* weight scale + index_add_ un-permute .......... C5/python/solution.py:158-160
* the C9 three-GEMM grouped expert compute ...... C9/python/solution.py:207-222
* the C9 tile metadata .......................... C9/python/solution.py:142-159

Two numeric modes:

``"ref"``  rounds to bf16 at every point where the reference's bf16 torch ops
           round (nn.Linear outputs, silu, the product, the weight scale and
           the index_add_ result), so it tracks the reference to within the
           summation order of the fp32 GEMM sums.
``"fp32"`` keeps every intermediate in fp32 (inputs are the same bf16 values);
           this is the tolerance target for the CUDA path
           (max|y - y_ref| / max|y_ref| <= 2e-2).

Parity of this restatement is pinned against the reference itself, run in
the build container on CPU; the fixtures and the script that produced them
live in ``tests/golden/``.

Tie rule.  ``torch.topk`` leaves the order of equal values implementation
defined; this oracle fixes "larger value first, lower expert id first among
equal values", which equals ``torch.sort(logits, descending=True,
stable=True)[:, :k]``.  The permutation is the stable one (records of one
expert keep their flat slot order n*k+j), which is what C6:152 and C8:181 use.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 helpers (bf16 held as uint16 bit patterns or as bf16-exact float32)
# ---------------------------------------------------------------------------


def bf16_bits_from_f32(a: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even) and return the uint16 bits."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def f32_from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """Widen uint16 bf16 bit patterns to float32 (exact)."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return f32_from_bf16_bits(bf16_bits_from_f32(a))


def _maybe_round(a: np.ndarray, mode: str) -> np.ndarray:
    return bf16_round(a) if mode == "ref" else a.astype(np.float32, copy=False)


# ---------------------------------------------------------------------------
# Router (C5:124-129)
# ---------------------------------------------------------------------------


def router_logits(x: np.ndarray, wr: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """``self.gate(x_flat)`` (C5:124): fp32-accumulated x @ Wr^T, rounded to bf16.

    ``bias`` (fp32, [E]) is added before the rounding; it stands for the
    skewed-routing bias of the expert-parallel workload (an ``nn.Linear``
    with ``bias=True`` in place of the reference's bias-free gate).
    """
    acc = x.astype(np.float32) @ wr.astype(np.float32).T
    if bias is not None:
        acc = acc + bias.astype(np.float32)[None, :]
    return bf16_round(acc)


def topk_ids(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """``torch.topk(router_logits, k)`` (C5:125) with the fixed tie rule.

    Returns (values [T,k] float32, ids [T,k] int64), values descending; equal
    values are ordered by ascending expert id.
    """
    order = np.argsort(-logits, axis=-1, kind="stable")[:, :k]
    vals = np.take_along_axis(logits, order, axis=-1)
    return vals.astype(np.float32), order.astype(np.int64)


def softmax_f32(v: np.ndarray) -> np.ndarray:
    m = v.max(axis=-1, keepdims=True)
    e = np.exp(v - m, dtype=np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def topk_weights(logits: np.ndarray, vals: np.ndarray, ids: np.ndarray,
                 norm_topk_prob: bool = True, mode: str = "ref") -> np.ndarray:
    """Top-k routing weights (C5:126-129).

    ``norm_topk_prob=True``: softmax over the k selected logits, which equals a
    softmax over all E followed by renormalising the top k.  Otherwise the
    softmax over all E gathered at the selected ids.  ``mode="ref"`` rounds the
    result to bf16 like the reference's bf16 ``F.softmax``.
    """
    if norm_topk_prob:
        w = softmax_f32(vals)
    else:
        w = np.take_along_axis(softmax_f32(logits), ids, axis=-1)
    return _maybe_round(w, mode)


# ---------------------------------------------------------------------------
# Sort / align (C5:131-138, C6:152-160, C9:142-159)
# ---------------------------------------------------------------------------


def sort_by_expert(ids_flat: np.ndarray, num_experts: int):
    """Stable argsort of the flat expert ids plus per-expert counts/offsets.

    Returns (perm, sorted_ids, counts, offsets): ``perm[p]`` is the flat slot
    index n*k+j of the p-th record in expert order; ``offsets`` has E+1
    entries with ``offsets[0] = 0`` (C6:159-160's ``F.pad(cumsum)``).
    """
    ids_flat = np.asarray(ids_flat, dtype=np.int64)
    perm = np.argsort(ids_flat, kind="stable").astype(np.int64)
    sorted_ids = ids_flat[perm]
    counts = np.bincount(ids_flat, minlength=num_experts).astype(np.int64)
    offsets = np.zeros(num_experts + 1, dtype=np.int64)
    np.cumsum(counts, out=offsets[1:])
    return perm, sorted_ids, counts, offsets


def tile_metadata(offsets: np.ndarray, block_m: int):
    """``_build_meta_data`` (C9:142-159): per M-tile its expert id and its
    tile index inside that expert, for tiles of ``block_m`` rows."""
    offsets = np.asarray(offsets, dtype=np.int64)
    counts = offsets[1:] - offsets[:-1]
    ntiles = (counts + block_m - 1) // block_m
    tile_expert = np.repeat(np.arange(len(counts), dtype=np.int64), ntiles)
    first = np.cumsum(ntiles) - ntiles
    tile_in_expert = np.arange(len(tile_expert), dtype=np.int64) - np.repeat(first, ntiles)
    return tile_expert, tile_in_expert


# ---------------------------------------------------------------------------
# Expert compute (C5:68-80, C9:207-222)
# ---------------------------------------------------------------------------


def silu_f32(a: np.ndarray) -> np.ndarray:
    a = a.astype(np.float32, copy=False)
    return (a / (np.float32(1.0) + np.exp(-a, dtype=np.float32))).astype(np.float32)


def swiglu_expert(xs: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray,
                  mode: str = "ref") -> np.ndarray:
    """``down(silu(gate(x)) * up(x))`` for one expert (C5:79-80)."""
    g = _maybe_round(xs @ wg.T, mode)
    u = _maybe_round(xs @ wu.T, mode)
    h = _maybe_round(_maybe_round(silu_f32(g), mode) * u, mode)
    return _maybe_round(h @ wd.T, mode)


def fused_moe_forward(sorted_x: np.ndarray, offsets: np.ndarray, w_gate: np.ndarray,
                      w_up: np.ndarray, w_down: np.ndarray, mode: str = "ref") -> np.ndarray:
    """The C9 grouped compute (C9:207-222): per expert e, rows
    ``offsets[e]:offsets[e+1]`` of ``sorted_x`` go through SwiGLU; the output is
    unweighted and still in sorted order.  Rows past ``offsets[E]`` stay zero
    (C9:180 allocates ``y`` with ``zeros``)."""
    M = sorted_x.shape[0]
    out = np.zeros((M, w_down.shape[1]), dtype=np.float32)
    xs_all = sorted_x.astype(np.float32)
    for e in range(w_gate.shape[0]):
        s, t = int(offsets[e]), int(offsets[e + 1])
        if s == t:
            continue
        out[s:t] = swiglu_expert(xs_all[s:t], w_gate[e].astype(np.float32),
                                 w_up[e].astype(np.float32), w_down[e].astype(np.float32), mode)
    return out


def index_add_rows(num_tokens: int, tok: np.ndarray, src: np.ndarray, mode: str = "ref") -> np.ndarray:
    """``y.index_add_(0, tok, src)`` into a zero ``y`` (C5:119,160).

    The reference's bf16 ``index_add_`` on CPU sums each token's rows in fp32
    and rounds once to bf16 (checked against torch in the build container), so
    ``"ref"`` mode is the fp32 sum rounded to bf16 and ``"fp32"`` mode the sum
    itself.
    """
    H = src.shape[1]
    y = np.zeros((num_tokens, H), dtype=np.float32)
    np.add.at(y, tok, src.astype(np.float32))
    return _maybe_round(y, mode)


def permuted_moe(x: np.ndarray, wr: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray,
                 w_down: np.ndarray, top_k: int, norm_topk_prob: bool = True,
                 mode: str = "ref", bias: np.ndarray | None = None,
                 logits: np.ndarray | None = None, ids: np.ndarray | None = None) -> dict:
    """``PermutedSparseMoE.forward`` (C5:108-161) on flat ``x[T,H]``.

    Returns a dict with every intermediate the CUDA path exposes: logits,
    ids, weights, perm, counts, offsets, tok (token of each sorted record) and
    y.  ``logits`` may be passed in to route on given bf16 logits (used to
    check routing bit-exactly against the CUDA router's own logits), and
    ``ids`` to force the selected experts (used where the reference broke a
    logit tie at the top-k boundary differently).
    """
    T = x.shape[0]
    E = wr.shape[0]
    xf = x.astype(np.float32)
    if logits is None:
        logits = router_logits(xf, wr, bias)
    if ids is None:
        vals, ids = topk_ids(logits, top_k)
    else:
        ids = np.asarray(ids, dtype=np.int64)
        vals = np.take_along_axis(logits, ids, axis=-1)
    w = topk_weights(logits, vals, ids, norm_topk_prob, mode)
    ids_flat = ids.reshape(-1)
    perm, sorted_ids, counts, offsets = sort_by_expert(ids_flat, E)
    tok = perm // top_k
    sorted_x = xf[tok]
    sorted_w = w.reshape(-1)[perm]
    out = fused_moe_forward(sorted_x, offsets, w_gate, w_up, w_down, mode)
    scaled = _maybe_round(out * sorted_w[:, None], mode)
    y = index_add_rows(T, tok, scaled, mode)
    return dict(logits=logits, vals=vals, ids=ids, weights=w, perm=perm,
                sorted_ids=sorted_ids, counts=counts, offsets=offsets, tok=tok,
                expert_out=out, y=y)


def rel_err(y: np.ndarray, y_ref: np.ndarray) -> float:
    """max|y - y_ref| / max|y_ref| — the output tolerance measure."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    den = float(np.abs(y_ref).max())
    return float(np.abs(y - y_ref).max()) / (den if den > 0 else 1.0)


# ---------------------------------------------------------------------------
# Seeded inputs (numpy PCG64: identical on every x86 host)
# ---------------------------------------------------------------------------


def make_inputs(T: int, H: int, I: int, E: int, seed: int = 0, wscale: float = 0.02,
                experts: bool = True) -> dict:
    """Seeded bf16 inputs of the benchmark's distribution, as uint16 bits.

    x ~ N(0,1); router weight Wr[E,H], w_gate/w_up[E,I,H] and w_down[E,H,I]
    ~ N(0, wscale).  Drawn in the fixed order x, Wr, w_gate, w_up, w_down from
    ``np.random.default_rng(seed)``.
    """
    rng = np.random.default_rng(seed)
    out = {}
    out["x"] = bf16_bits_from_f32(rng.standard_normal((T, H), dtype=np.float32))
    out["wr"] = bf16_bits_from_f32(rng.standard_normal((E, H), dtype=np.float32) * np.float32(wscale))
    if experts:
        out["w_gate"] = bf16_bits_from_f32(rng.standard_normal((E, I, H), dtype=np.float32) * np.float32(wscale))
        out["w_up"] = bf16_bits_from_f32(rng.standard_normal((E, I, H), dtype=np.float32) * np.float32(wscale))
        out["w_down"] = bf16_bits_from_f32(rng.standard_normal((E, H, I), dtype=np.float32) * np.float32(wscale))
    return out


def zipf_bias(E: int, s: float = 1.2) -> np.ndarray:
    """Skewed-routing bias b_e = -s * ln(e + 1), added to the fp32 router
    logits before bf16 rounding (the expert-parallel imbalance workload)."""
    return (-s * np.log(np.arange(E, dtype=np.float64) + 1.0)).astype(np.float32)
