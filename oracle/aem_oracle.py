"""CPU oracle for the AetherMoE MoE-layer hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it.  The product path (``aethermoe_b200``) never calls into it and
fails loudly when its CUDA library is missing.

Every function restates, in NumPy, the algorithm of one reference function;
the docstrings cite the reference file:line it follows (paths are relative to
the AetherMoE project root).  Parity is pinned in two ways (see
``tests/golden/make_golden.py``):

* golden vectors produced by importing the reference's own
  ``prototype/math_proto.py`` and ``validation/pytorch_reference.py``;
* the reference's C++ ``Router`` compiled from its header into
  ``oracle/_ref`` (``oracle/Makefile``), run on the same seeded batches.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "gating_logits_seq", "topk_strict", "softmax_selected", "fused_gating",
    "reference_gating", "quantize_int8", "dequantize_int8", "qgemm",
    "capacity_assign", "moe_units", "moe_route", "bf16_round",
    "moe_layer", "moe_layer_rows", "ep_local_counts", "ep_slot_bases",
    "zipf_bias", "default_capacity", "certified_fast_logits",
]


# ----------------------------------------------------------------------------
# Gating  (A1/A2)
# ----------------------------------------------------------------------------

def gating_logits_seq(hidden, gate_weight, gate_bias):
    """Logits with the arithmetic of ``fused_kernel_simulation``.

    Follows ``prototype/math_proto.py:33-34``: every product
    ``hidden[n,d]*gate_weight[d,e]`` is a float32 product, the products are
    summed in float32 in increasing ``d`` order (Python ``sum`` starting from
    the integer 0), and the float32 bias is added last.  NumPy float32
    elementwise ops never fuse a multiply and an add, so this vectorised
    form is bit-identical to the reference loop.
    """
    h = np.ascontiguousarray(hidden, dtype=np.float32)
    w = np.ascontiguousarray(gate_weight, dtype=np.float32)
    b = np.asarray(gate_bias, dtype=np.float32).reshape(-1)
    n, d = h.shape
    d2, e = w.shape
    assert d == d2 and b.shape[0] == e
    ht = np.ascontiguousarray(h.T)  # rows of ht are columns of h: contiguous per d
    acc = np.zeros((n, e), dtype=np.float32)
    tmp = np.empty((n, e), dtype=np.float32)
    for k in range(d):
        np.multiply(ht[k][:, None], w[k][None, :], out=tmp)
        np.add(acc, tmp, out=acc)
    return (acc + b[None, :]).astype(np.float32)


def topk_strict(logits, k, return_values=False):
    """Iterative strict-``>`` max extraction, ties to the lowest expert id.

    Follows the kernel's selection loop ``src/kernels/fused_gating_metal.py:281-293``
    and its NumPy twin ``prototype/math_proto.py:38-43``: ``np.argmax`` (the
    lowest index of equal maxima; the first NaN when the row holds one), then
    the winner is overwritten with ``-inf`` -- it is not removed, so a row with
    fewer than ``k`` entries above ``-inf`` selects its lowest ``-inf`` index
    again.  Returns int64 ``[N, k]`` ordered by descending logit and, with
    ``return_values``, the float32 values recorded at each selection (the
    row's current entry, as ``math_proto.py:40`` records ``local[best_idx]``).
    """
    local = np.array(logits, dtype=np.float32, copy=True)
    n, e = local.shape
    assert 0 <= k <= e
    out = np.zeros((n, k), dtype=np.int64)
    vals = np.zeros((n, k), dtype=np.float32)
    rows = np.arange(n)
    for kk in range(k):
        best = np.argmax(local, axis=1)
        out[:, kk] = best
        vals[:, kk] = local[rows, best]
        local[rows, best] = -np.inf
    return (out, vals) if return_values else out


def softmax_selected(vals):
    """Softmax over the selected logits with max subtraction, in float32.

    Follows ``prototype/math_proto.py:44-47`` (and the kernel tail
    ``src/kernels/fused_gating_metal.py:295-305``).
    """
    v = np.asarray(vals, dtype=np.float32)
    m = v.max(axis=-1, keepdims=True)
    e = np.exp(v - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def fused_gating(hidden, gate_weight, gate_bias, k, extra=0):
    """Oracle of the fused gating kernel: ``(idx int32 [N,k+extra], val f32 [N,k])``.

    ``extra`` additional indices (the next choices after the top-k, in the
    same descending order) are returned for capacity rerouting; they receive
    no softmax weight.  ``extra`` is clipped so that ``k+extra <= E``.
    """
    logits = gating_logits_seq(hidden, gate_weight, gate_bias)
    e = logits.shape[1]
    ksel = min(k + extra, e)
    idx, sel = topk_strict(logits, ksel, return_values=True)
    return idx.astype(np.int32), softmax_selected(sel[:, :k])


def reference_gating(hidden, gate_weight, gate_bias, k):
    """``prototype/math_proto.py:8-17`` with a stable descending sort.

    The reference sorts with ``np.argsort(-logits)`` (default quicksort,
    tie order unspecified); a stable sort gives the lowest id first on ties,
    the contract of the kernel.  Logits come from BLAS (summation order
    unspecified), so this is the VALUE oracle; ``fused_gating`` is the
    index oracle.
    """
    logits = (np.asarray(hidden, np.float32) @ np.asarray(gate_weight, np.float32)
              + np.asarray(gate_bias, np.float32))
    order = np.argsort(-logits, axis=-1, kind="stable")
    idx = order[:, :k]
    sel = np.take_along_axis(logits, idx, axis=-1)
    return idx, softmax_selected(sel)


def certified_rows(hidden, gate_weight, gate_bias, k):
    """Rows whose top-k set is decided beyond float32 rounding error.

    A row is certified when the gap between its k-th and (k+1)-th float64
    logits exceeds twice the forward error bound of a float32 dot product,
    ``gamma_D * sum_d |x_d w_de|`` with ``gamma_D = D u / (1 - D u)``,
    ``u = 2**-24``.  Used only for comparisons against implementations whose
    summation order differs from the sequential one (BLAS, torch).
    """
    h = np.asarray(hidden, np.float64)
    w = np.asarray(gate_weight, np.float64)
    b = np.asarray(gate_bias, np.float64)
    n, d = h.shape
    e = w.shape[1]
    lg = h @ w + b
    u = 2.0 ** -24
    gam = (d + 1) * u / (1 - (d + 1) * u)
    bound = gam * (np.abs(h) @ np.abs(w) + np.abs(b))
    if k >= e:
        return np.ones(n, dtype=bool)
    order = np.argsort(-lg, axis=1, kind="stable")
    kth = np.take_along_axis(lg, order[:, k - 1:k], 1)[:, 0]
    nxt = np.take_along_axis(lg, order[:, k:k + 1], 1)[:, 0]
    bk = np.take_along_axis(bound, order[:, k - 1:k], 1)[:, 0]
    bn = np.take_along_axis(bound, order[:, k:k + 1], 1)[:, 0]
    return (kth - nxt) > 2.0 * (bk + bn)


def _fma32(a, b, c):
    """float32 fused multiply-add a*b + c with one rounding: the float32
    product is exact in float64 and the float64 sum is rounded once to
    float32 (a double rounding that differs from a true single rounding only
    at float64 ties -- far inside the bound's margin)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def certified_fast_logits(hidden, gate_weight, gate_bias, parts=1, block=64):
    """Fast logits and their certified bound, the arithmetic of the CERTIFIED
    gating kernels (this library's own mode: the reference has only the
    sequential form of ``prototype/math_proto.py:33-34``).

    d is cut into ``parts`` contiguous parts of whole ``block``-wide blocks;
    each part is a chain of float32 fused multiply-adds from zero; after each
    block ``Q += block |P| + (block + 1) |x_block| |w_block|``; the parts are
    then added in order with ``Q += len(part) |P_start|`` and ``Qc += |P_start|
    + |S_part|``, the bias added last.  Returns ``(F, B)`` float32 ``[N, E]``
    with ``B = 4 u (Q + Qc + |F| + |b|)``, ``u = 2**-24``: the bound on the
    distance from the sequential logits (``gating_logits_seq``).
    """
    h = np.ascontiguousarray(hidden, dtype=np.float32)
    w = np.ascontiguousarray(gate_weight, dtype=np.float32)
    b = np.asarray(gate_bias, dtype=np.float32).reshape(-1)
    n, d = h.shape
    e = w.shape[1]
    nblk = -(-d // block)
    dpad = nblk * block
    hp = np.zeros((n, dpad), np.float32)
    hp[:, :d] = h
    wp = np.zeros((dpad, e), np.float32)
    wp[:d] = w
    bpp = -(-nblk // parts)
    xn = np.sqrt(np.square(hp.reshape(n, nblk, block).astype(np.float64)).sum(2)).astype(np.float32)
    wn = np.sqrt(np.square(wp.reshape(nblk, block, e).astype(np.float64)).sum(1)).astype(np.float32)
    run = np.zeros((n, e), np.float32)
    Q = np.zeros((n, e), np.float64)
    Qc = np.zeros((n, e), np.float64)
    for p in range(parts):
        acc = np.zeros((n, e), np.float32)
        q = np.zeros((n, e), np.float64)
        for blk in range(p * bpp, min(nblk, (p + 1) * bpp)):
            for dd in range(blk * block, (blk + 1) * block):
                acc = _fma32(hp[:, dd][:, None], wp[dd][None, :], acc)
            q += block * np.abs(acc.astype(np.float64)) + (block + 1) * (
                xn[:, blk][:, None].astype(np.float64) * wn[blk][None, :])
        Q += q + block * bpp * np.abs(run.astype(np.float64))
        Qc += np.abs(run.astype(np.float64)) + np.abs(acc.astype(np.float64))
        run = (run + acc).astype(np.float32)
    f = (run + b[None, :]).astype(np.float32)
    u = 2.0 ** -24
    bound = (4 * u * (Q + Qc + np.abs(f) + np.abs(b)[None, :])).astype(np.float32)
    return f, bound


# ----------------------------------------------------------------------------
# INT8 weight-only quantisation and GEMM  (A3/A4/A5)
# ----------------------------------------------------------------------------

def quantize_int8(weight_fp32):
    """Per-output-column symmetric INT8 quantisation, bit-exact float32.

    Follows ``prototype/math_proto.py:52-66`` and ``src/kernels/quantized_gemm.py:70-76``:
    ``scale = max(max_k |w[k,n]| / 127, 1e-12)`` in float32 and
    ``q = clip(round_half_even(w / scale), -127, 127)``.
    Returns ``(q int8 [K,N], scale f32 [1,N])``.
    """
    w = np.asarray(weight_fp32, dtype=np.float32)
    scale = np.abs(w).max(axis=0, keepdims=True) / np.float32(127.0)
    scale = np.maximum(scale, np.float32(1e-12)).astype(np.float32)
    q = np.round(w / scale).clip(-127, 127).astype(np.int8)
    return q, scale


def dequantize_int8(q, scale):
    """``prototype/math_proto.py:68-69``: ``q.astype(f32) * scale``."""
    return np.asarray(q).astype(np.float32) * np.asarray(scale, np.float32)


def qgemm(x, q, scale):
    """``out[m,n] = sum_k x[m,k] * (q[k,n]*scale[n])`` in float64.

    The float32 dequantised weight follows ``prototype/math_proto.py:83``
    (``q * scale`` per element); the reduction is float64, i.e. the exact
    value the reference's float32 kernels (``quantized_gemm.py:129-132``,
    ``math_proto.py:71-86``) approximate.
    """
    w = dequantize_int8(q, scale).astype(np.float64)
    return np.asarray(x, np.float64) @ w


# ----------------------------------------------------------------------------
# Capacity-ceiling routing  (A6)
# ----------------------------------------------------------------------------

def capacity_assign(primary, secondary, batch_position, capacity):
    """Effective expert per token under the capacity ceiling.

    Follows ``Router::assign_effective_experts`` in
    ``src/orchestration/router.hpp:249-266`` (and its independent test
    restatement ``tests/test_orchestration.cpp:187-205``): tokens are
    grouped by primary expert, each group is ranked by ``batch_position``;
    rank < capacity keeps the primary, the rest take their own secondary
    (one hop, the secondary is not capacity-checked, ``router.hpp:21-27``).
    ``capacity=None`` means unlimited (``router.hpp:50``).
    """
    p = np.asarray(primary, dtype=np.int64)
    s = np.asarray(secondary, dtype=np.int64)
    pos = np.asarray(batch_position, dtype=np.int64)
    n = p.shape[0]
    if capacity is None or n == 0:
        return p.astype(np.int32).copy()
    order = np.argsort(pos, kind="stable")           # by batch_position
    po = p[order]
    grp = np.argsort(po, kind="stable")              # stable: keeps position order
    sorted_p = po[grp]
    starts = np.r_[0, np.flatnonzero(np.diff(sorted_p)) + 1]
    lens = np.diff(np.r_[starts, n])
    rank_sorted = np.arange(n) - np.repeat(starts, lens)
    rank = np.empty(n, dtype=np.int64)
    rank[order[grp]] = rank_sorted
    eff = np.where(rank < capacity, p, s)
    return eff.astype(np.int32)


def default_capacity(tokens, k, experts, factor=1.25):
    """``ceil(factor * tokens * k / experts)`` -- the expert-parallel capacity."""
    return int(math.ceil(factor * tokens * k / experts))


def moe_units(idx_ext, k, num_experts):
    """Flatten ``(token, slot)`` pairs into routing units, slot-major.

    Unit ``u = j*T + t`` has ``batch_position = u``, ``primary = idx[t,j]``
    and ``secondary = idx[t,k]`` (the token's (k+1)-th choice; when
    ``k == E`` there is none and the secondary is the primary).  For k=1
    this is exactly the reference's ``RoutedToken`` contract
    (``src/orchestration/routed_token.hpp:24-41``): primary = best expert,
    secondary = second choice.  Returns ``(primary, secondary, position,
    token, slot)`` int arrays of length ``T*k``.
    """
    idx = np.asarray(idx_ext)
    t = idx.shape[0]
    prim = idx[:, :k].T.reshape(-1).astype(np.int32)
    if k < num_experts:
        sec = np.tile(idx[:, k], k).astype(np.int32)
    else:
        sec = prim.copy()
    pos = np.arange(t * k, dtype=np.int64)
    tok = np.tile(np.arange(t, dtype=np.int32), k)
    slot = np.repeat(np.arange(k, dtype=np.int32), t)
    return prim, sec, pos, tok, slot


def moe_route(idx_ext, k, num_experts, capacity):
    """Effective expert of every unit of ``moe_units`` (slot-major order)."""
    prim, sec, pos, _, _ = moe_units(idx_ext, k, num_experts)
    return capacity_assign(prim, sec, pos, capacity)


def ep_local_counts(idx_ext, k, num_experts):
    """Per-(slot, expert) primary counts of one rank's tokens: ``int64 [k, E]``."""
    idx = np.asarray(idx_ext)
    out = np.zeros((k, num_experts), dtype=np.int64)
    for j in range(k):
        out[j] = np.bincount(idx[:, j], minlength=num_experts)
    return out


def ep_slot_bases(all_counts, rank):
    """Global rank offset of each (slot, expert) group for one rank.

    With tokens split contiguously across ranks and units ordered slot-major
    by global batch position, the units of slot ``j`` on rank ``r`` come
    after every unit of slots ``< j`` (all ranks) and after slot ``j`` of
    ranks ``< r``.  ``all_counts`` is ``[R, k, E]``; returns ``int64 [k, E]``.
    """
    c = np.asarray(all_counts, dtype=np.int64)
    per_slot = c.sum(axis=0)                                   # [k, E]
    before_slots = np.cumsum(per_slot, axis=0) - per_slot      # exclusive over j
    before_ranks = c[:rank].sum(axis=0)                        # [k, E]
    return before_slots + before_ranks


# ----------------------------------------------------------------------------
# MoE layer composed from the pieces
# ----------------------------------------------------------------------------

def bf16_round(a):
    """Round float32 values to bfloat16 (round-to-nearest-even), as float32."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(f)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def zipf_bias(num_experts, s=1.1):
    """Gate bias ``b_e = log p_e`` with ``p_e proportional to (e+1)^-s``."""
    p = (np.arange(num_experts, dtype=np.float64) + 1.0) ** (-s)
    p /= p.sum()
    return np.log(p).astype(np.float32)


def _expert_rows(xrow, qup, sup, qdn, sdn, hidden="bf16"):
    h = xrow.astype(np.float64) @ dequantize_int8(qup, sup).astype(np.float64)
    h = np.maximum(h, 0.0)
    if hidden == "bf16":
        h = bf16_round(h.astype(np.float32)).astype(np.float64)
    return h @ dequantize_int8(qdn, sdn).astype(np.float64)


def moe_layer(x, gate_w, gate_b, k, q_up, s_up, q_down, s_down, capacity=None, hidden="bf16"):
    """Oracle of one MoE layer: gating -> capacity routing -> expert FFN -> combine.

    ``x`` [T,d] float32 (the values the layer receives: float32 inputs as
    they are, bfloat16 inputs as their float32 values); ``q_up[e]`` [d,ffn]
    int8 with ``s_up[e]`` [1,ffn]; ``q_down[e]`` [ffn,d] with ``s_down[e]``
    [1,d].  The expert FFN is ``relu(x @ deq(q_up)) @ deq(q_down)`` in float64
    -- the float32-activation GEMM contract of
    ``src/kernels/quantized_gemm.py:184-226`` / ``prototype/math_proto.py:71-86``
    evaluated exactly -- with the hidden activation rounded to bfloat16 only
    when ``hidden == "bf16"`` (a layer that stores it in bf16).  The layer
    output is ``sum_j val[t,j] * y[t,j]``.
    Returns ``(out f64 [T,d], idx int32 [T,k(+1)], val f32 [T,k], eff int32 [T*k])``.
    """
    x = np.asarray(x, np.float32)
    t = x.shape[0]
    e = gate_w.shape[1]
    idx, val = fused_gating(x, gate_w, gate_b, k, extra=1)
    eff = moe_route(idx, k, e, capacity)
    out = np.zeros((t, x.shape[1]), dtype=np.float64)
    _, _, _, tok, slot = moe_units(idx, k, e)
    for ex in range(e):
        sel = np.flatnonzero(eff == ex)
        if sel.size == 0:
            continue
        y = _expert_rows(x[tok[sel]], q_up[ex], s_up[ex], q_down[ex], s_down[ex], hidden)
        w = val[tok[sel], slot[sel]].astype(np.float64)[:, None]
        np.add.at(out, tok[sel], w * y)
    return out, idx, val, eff


def moe_layer_rows(rows, x, idx, val, eff, k, q_up, s_up, q_down, s_down, hidden="bf16"):
    """Layer output for a subset of token ``rows`` given the routing decision.

    Used to check sampled rows of full-size runs without the whole layer;
    each expert's weights are dequantised once for all the rows it serves.
    """
    rows = np.asarray(rows)
    t = x.shape[0]
    out = np.zeros((len(rows), x.shape[1]), dtype=np.float64)
    unit_row = np.repeat(np.arange(len(rows)), k)
    unit_slot = np.tile(np.arange(k), len(rows))
    unit_tok = rows[unit_row]
    unit_eff = np.asarray(eff)[unit_slot * t + unit_tok]
    for ex in np.unique(unit_eff):
        sel = np.flatnonzero(unit_eff == ex)
        y = _expert_rows(np.asarray(x, np.float32)[unit_tok[sel]], q_up[ex], s_up[ex],
                         q_down[ex], s_down[ex], hidden)
        w = np.asarray(val)[unit_tok[sel], unit_slot[sel]].astype(np.float64)[:, None]
        np.add.at(out, unit_row[sel], w * y)
    return out
