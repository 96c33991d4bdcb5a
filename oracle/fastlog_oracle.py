"""CPU oracle for MiniKG's relation-typed sparse hop (TEST INFRASTRUCTURE ONLY).

This module restates, in numpy, the reference algorithm of the path behind
``src/fastlog_bridge.py`` in majh3/miniKG_dev.  It is the checker for the CUDA
product and the timed CPU baseline; the product never imports it.  Only the
test-suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may call it.

Parity status: PINNED.  ``tests/golden/make_golden.py`` runs the reference's own
Python code (CPU, one torch thread) on seeded inputs and commits the outputs as
fixtures; ``tests/test_oracle_golden.py`` checks this module against them.

Arithmetic follows the reference step by step:

* message value ``v = (sv * w) * m`` in float32, ``m = bool(mask[e]) * score(e)``
  with ``score = edge_weight[e]`` (score mode) or ``sigmoid(edge_weight[e] * scale)``
  (src/fastlog_kernel/source/fastlog.cu:2300-2318);
* the per-entry edge cap with the 256-bucket histogram and in-order threshold
  groups (fastlog.cu:2092-2195, 2273-2298);
* coalescing by the int64 key ``b*L*E + l*E + e`` with a stable sort and an
  in-order float32 ``scatter_add_`` (src/fastlog_kernel/fastlog_kernel.py:81-104);
* the max coalesce with argmax ties broken by the smallest original fact id,
  then the smallest raw-message position (fastlog_kernel.py:107-150);
* backward kernels and the edge-score gradient (fastlog.cu:2551-2676,
  fastlog_kernel.py:153-190, 242-261, 1032-1098);
* the bridge / proof-loop reducers (src/fastlog_bridge.py:17-42,
  src/model_mmDRUM_kernel_sp.py:39-270, drum.py:31-80, proof.py:467-649,
  decode_core.py:350-363).

Sums that the reference performs with ``scatter_add_`` / ``index_add_`` /
``index_put_(accumulate=True)`` on CPU are sequential in index order; this module
reproduces them with ``np.add.at`` (sequential, float32).

``float64_arithmetic()`` reruns the same restatement with every value held in float64
(the per-hop cap decisions stay on the float32 rule weights, as the reference decides
them): the exact value of the reference's computation, to which its own float32 results
are rounded approximations.  The sum-loop gradient tests measure the CUDA path against
it, because over several hops the reference's own float32 rounding already moves its
gradients further from that value than the fp32 tolerance (measured in
``tests/test_oracle_golden.py``).

A sparse ``[B, L, E]`` tensor is a pair ``(keys, vals)``: sorted unique int64 keys
``(b*L + l)*E + e`` and float32 values.
"""
from __future__ import annotations

import contextlib

import numpy as np

F32 = np.float32  # arithmetic type of the restatement (float64 inside float64_arithmetic())
NUM_BUCKETS = 256
UNCAPPED = 1 << 60


@contextlib.contextmanager
def float64_arithmetic():
    """Run the restatement with float64 values and sums (test infrastructure: the exact
    value of the reference computation for tolerance checks).  Not thread-safe."""
    global F32
    old = F32
    F32 = np.float64
    try:
        yield
    finally:
        F32 = old


# ----------------------------------------------------------------------------
# graph / CSR build  (fastlog_kernel.py:346-411, fastlog.cpp:9-16)
# ----------------------------------------------------------------------------

def ind2ptr(index: np.ndarray, size: int) -> np.ndarray:
    """Row pointer from sorted row ids (fastlog.cpp:9-16, fastlog_kernel.py:346-351)."""
    cnt = np.bincount(np.asarray(index, dtype=np.int64), minlength=size)[:size]
    ptr = np.zeros(size + 1, dtype=np.int64)
    np.cumsum(cnt, out=ptr[1:])
    ptr[-1] = index.shape[0]
    return ptr


def build_group_metadata(sorted_rows, sorted_rels, num_nodes):
    """(row_group_ptr i32, group_rel i16, group_edge_start i32, group_edge_count i32)
    per fastlog_kernel.py:354-368."""
    n = sorted_rows.shape[0]
    if n == 0:
        return (ind2ptr(np.empty(0, np.int64), num_nodes).astype(np.int32),
                np.empty(0, np.int16), np.empty(0, np.int32), np.empty(0, np.int32))
    starts = np.ones(n, dtype=bool)
    starts[1:] = (sorted_rows[1:] != sorted_rows[:-1]) | (sorted_rels[1:] != sorted_rels[:-1])
    gstart = np.nonzero(starts)[0]
    grows = sorted_rows[gstart]
    grel = sorted_rels[gstart].astype(np.int16)
    nxt = np.concatenate([gstart[1:], [n]])
    gcnt = (nxt - gstart).astype(np.int32)
    rgp = ind2ptr(grows, num_nodes).astype(np.int32)
    return rgp, grel, gstart.astype(np.int32), gcnt


def build_csr_structure(row, col, rel, num_nodes):
    """The reference 16-tuple (fastlog_kernel.py:371-411), stable (row, rel, fact id) order.

    Returns (ori_row_ptr, ori_col_ind, ori_r_ind, ori_order,
             inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
             ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
             inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count).
    """
    row = np.asarray(row, dtype=np.int64)
    col = np.asarray(col, dtype=np.int64)
    rel = np.asarray(rel, dtype=np.int64)
    rel_base = int(rel.max()) + 1 if rel.shape[0] else 1
    out = []
    groups = []
    for src, dst in ((row, col), (col, row)):
        order = np.argsort(src * rel_base + rel, kind="stable")
        s_rows = src[order]
        s_rel = rel[order]
        out += [ind2ptr(s_rows, num_nodes).astype(np.int32), dst[order].astype(np.int32),
                s_rel.astype(np.int16), order.astype(np.int32)]
        groups += list(build_group_metadata(s_rows, s_rel, num_nodes))
    return tuple(out + groups)


# ----------------------------------------------------------------------------
# per-message factors
# ----------------------------------------------------------------------------

def message_factor(edge_ids, mask, edge_weight, is_score: bool, scale: float) -> np.ndarray:
    """``m = bool(mask[e]) * score(e)`` (fastlog.cu:2303-2309).

    ``mask`` of one element broadcasts to every fact (the reference passes a 0-d ones
    tensor for huge graphs, proof.py:546-550).  ``edge_weight`` None/empty means no
    score factor.
    """
    edge_ids = np.asarray(edge_ids, dtype=np.int64)
    mask = np.asarray(mask)
    if mask.size == 1:
        m = np.full(edge_ids.shape[0], F32(1.0) if bool(mask.reshape(-1)[0]) else F32(0.0), dtype=F32)
    else:
        m = (mask.reshape(-1)[edge_ids] != 0).astype(F32)
    if edge_weight is not None and np.asarray(edge_weight).size > 0:
        ew = np.asarray(edge_weight, dtype=F32).reshape(-1)[edge_ids]
        if is_score:
            score = ew
        else:
            score = sigmoid_f32(ew * F32(scale))
        m = (m * score).astype(F32)
    return m


def sigmoid_f32(x: np.ndarray) -> np.ndarray:
    """float32 ``1 / (1 + exp(-x))`` rounded from float64."""
    return (1.0 / (1.0 + np.exp(-np.asarray(x, dtype=np.float64)))).astype(F32)


def bucketize(x: np.ndarray) -> np.ndarray:
    """``min(max(int(x * 255.f), 0), 255)`` (fastlog.cu:16-20)."""
    y = np.asarray(x, dtype=np.float32) * np.float32(NUM_BUCKETS - 1)  # float32 in every mode
    y = np.clip(y, -1.0, 256.0)
    return np.clip(np.trunc(y).astype(np.int64), 0, NUM_BUCKETS - 1)


def _seg_exclusive_cumsum(vals: np.ndarray, seg: np.ndarray) -> np.ndarray:
    """Exclusive cumulative sum of int ``vals`` restarting at every change of sorted ``seg``."""
    if vals.shape[0] == 0:
        return vals.copy()
    c = np.cumsum(vals)
    starts = np.ones(seg.shape[0], dtype=bool)
    starts[1:] = seg[1:] != seg[:-1]
    base = np.maximum.accumulate(np.where(starts, c - vals, 0))
    return c - vals - base


# ----------------------------------------------------------------------------
# one hop: expansion of raw messages (fastlog.cu:2114-2323, 2526-2549)
# ----------------------------------------------------------------------------

def group_takes(sp_b, sp_l, sp_e, w, row_group_ptr, group_rel, group_edge_count,
                rel_offset: int, cap: int):
    """Per (entry, group) number of taken edges under the edge cap.

    Returns (entry_of_group, group_index, take, weight) in entry → group order.
    The threshold-bucket rule: groups in buckets above the threshold take all of
    their edges, below take none, and threshold-bucket groups take, in group
    order, ``clamp(remain - taken_before, 0, count)`` (fastlog.cu:2092-2112,
    2167-2194, 2273-2298).
    """
    F = sp_e.shape[0]
    gs = row_group_ptr[sp_e].astype(np.int64)
    ge = row_group_ptr[sp_e + 1].astype(np.int64)
    ng = ge - gs
    tot_groups = int(ng.sum())
    eog = np.repeat(np.arange(F, dtype=np.int64), ng)
    cum = np.zeros(F + 1, dtype=np.int64)
    np.cumsum(ng, out=cum[1:])
    gidx = gs[eog] + (np.arange(tot_groups, dtype=np.int64) - cum[eog])
    rel = group_rel[gidx].astype(np.int64)
    cnt = group_edge_count[gidx].astype(np.int64)
    wv = w[sp_b[eog], sp_l[eog], rel_offset + rel].astype(F32)
    take = cnt.copy()
    total = np.bincount(eog, weights=cnt, minlength=F).astype(np.int64) if tot_groups else np.zeros(F, np.int64)
    capped = total > cap
    if capped.any():
        bkt = bucketize(wv)
        cap_ids = np.nonzero(capped)[0]
        slot = np.full(F, -1, dtype=np.int64)
        slot[cap_ids] = np.arange(cap_ids.shape[0])
        gsel = capped[eog]
        hist = np.zeros((cap_ids.shape[0], NUM_BUCKETS), dtype=np.int64)
        np.add.at(hist, (slot[eog[gsel]], bkt[gsel]), cnt[gsel])
        desc = hist[:, ::-1]
        cs = np.cumsum(desc, axis=1)
        hit = cs >= cap
        first = np.argmax(hit, axis=1)
        tb = (NUM_BUCKETS - 1) - first
        before = cs[np.arange(cs.shape[0]), first] - desc[np.arange(cs.shape[0]), first]
        remain = cap - before
        e_tb = np.full(F, -1, dtype=np.int64)
        e_rem = np.zeros(F, dtype=np.int64)
        e_tb[cap_ids] = tb
        e_rem[cap_ids] = remain
        g_tb = e_tb[eog]
        is_tb = gsel & (bkt == g_tb)
        prior = _seg_exclusive_cumsum(np.where(is_tb, cnt, 0), eog)
        t_tb = np.clip(e_rem[eog] - prior, 0, cnt)
        take = np.where(~gsel, cnt, np.where(bkt > g_tb, cnt, np.where(bkt < g_tb, 0, t_tb)))
    return eog, gidx, take, wv


def expand_direction(sp_b, sp_l, sp_e, sp_v, w, row_group_ptr, group_rel, group_edge_start,
                     group_edge_count, col_ind, order, mask, edge_weight, is_score, scale,
                     rel_offset: int, cap: int):
    """Raw messages of one direction in reference order (entry → group → CSR position).

    Returns dict with b, l, e (int64), v (f32), entry (int64), rel (int16 relation id
    without offset), m (f32), edge (int64 original fact id).  Zero-``m`` messages are
    kept, as the CUDA fill kernel does (fastlog.cu:2300-2318).
    """
    eog, gidx, take, wv = group_takes(sp_b, sp_l, sp_e, w, row_group_ptr, group_rel,
                                      group_edge_count, rel_offset, cap)
    valid = take > 0
    vg = np.nonzero(valid)[0]
    vt = take[vg]
    M = int(vt.sum())
    msg_g = np.repeat(vg, vt)
    cum = np.zeros(vg.shape[0] + 1, dtype=np.int64)
    np.cumsum(vt, out=cum[1:])
    local = np.arange(M, dtype=np.int64) - np.repeat(cum[:-1], vt)
    pos = group_edge_start[gidx[msg_g]].astype(np.int64) + local
    entry = eog[msg_g]
    edge = order[pos].astype(np.int64)
    m = message_factor(edge, mask, edge_weight, is_score, scale)
    v = ((sp_v[entry].astype(F32) * wv[msg_g]) * m).astype(F32)
    return dict(b=sp_b[entry].astype(np.int64), l=sp_l[entry].astype(np.int64),
                e=col_ind[pos].astype(np.int64), v=v, entry=entry,
                rel=group_rel[gidx[msg_g]].astype(np.int16), m=m, edge=edge)


# ----------------------------------------------------------------------------
# coalescing (fastlog_kernel.py:81-150)
# ----------------------------------------------------------------------------

def keys3(b, l, e, L, E):
    return (np.asarray(b, np.int64) * L + np.asarray(l, np.int64)) * E + np.asarray(e, np.int64)


def split3(keys, L, E):
    keys = np.asarray(keys, np.int64)
    return keys // (L * E), (keys % (L * E)) // E, keys % E


def coalesce_sum(keys, vals):
    """Sorted unique keys + in-order float32 sums (``_coalesce_sparse3d_reduce`` sum)."""
    keys = np.asarray(keys, np.int64)
    if keys.shape[0] == 0:
        return np.empty(0, np.int64), np.empty(0, F32)
    order = np.argsort(keys, kind="stable")
    sk = keys[order]
    uk, inv = np.unique(sk, return_inverse=True)
    out = np.zeros(uk.shape[0], dtype=F32)
    np.add.at(out, inv, np.asarray(vals, F32)[order])
    return uk, out


def coalesce_max_with_arg(keys, vals, tie):
    """Max per key; argmax = smallest ``tie`` among maxima, then smallest raw position
    (``_coalesce_sparse3d_max_with_arg``, fastlog_kernel.py:107-150).

    Returns (keys, max values, raw_arg int64 indices into the raw arrays).
    """
    keys = np.asarray(keys, np.int64)
    if keys.shape[0] == 0:
        return np.empty(0, np.int64), np.empty(0, F32), np.empty(0, np.int64)
    vals = np.asarray(vals, F32)
    tie = np.asarray(tie, np.int64)
    pos = np.arange(keys.shape[0], dtype=np.int64)
    # key asc, value desc, tie asc, raw position asc
    order = np.lexsort((pos, tie, -vals.astype(np.float64), keys))
    sk = keys[order]
    first = np.ones(sk.shape[0], dtype=bool)
    first[1:] = sk[1:] != sk[:-1]
    win = order[first]
    return keys[win], vals[win], win.astype(np.int64)


# ----------------------------------------------------------------------------
# the per-hop op  (FastLogFunctionSparse3DTopK, fastlog_kernel.py:900-1107)
# ----------------------------------------------------------------------------

def sparse3d_forward(sp_b, sp_l, sp_e, sp_v, w, csr, mask, edge_weight, B, L, E, r_size,
                     wot_i=False, cap=UNCAPPED, agg_mode=0, is_score=False, scale=1.0):
    """One hop.  Returns a dict with coalesced ``ori``, ``inv``, ``ind`` (keys, vals), the
    raw message dicts, and for ``agg_mode == 1`` the argmax raw positions."""
    sp_b = np.asarray(sp_b, np.int64); sp_l = np.asarray(sp_l, np.int64)
    sp_e = np.asarray(sp_e, np.int64); sp_v = np.asarray(sp_v, F32)
    w = np.asarray(w, F32)
    n = w.shape[2]
    (_, ori_col, _, ori_order, _, inv_col, _, inv_order,
     org_ptr, org_rel, org_start, org_cnt, irg_ptr, irg_rel, irg_start, irg_cnt) = csr
    raw_ori = expand_direction(sp_b, sp_l, sp_e, sp_v, w, org_ptr, org_rel, org_start, org_cnt,
                               ori_col, ori_order, mask, edge_weight, is_score, scale, 0, cap)
    raw_inv = expand_direction(sp_b, sp_l, sp_e, sp_v, w, irg_ptr, irg_rel, irg_start, irg_cnt,
                               inv_col, inv_order, mask, edge_weight, is_score, scale, r_size, cap)
    if wot_i:
        ind_v = np.zeros(sp_v.shape[0], F32)
    else:
        ind_v = (sp_v * w[sp_b, sp_l, n - 1]).astype(F32)
    out = dict(raw_ori=raw_ori, raw_inv=raw_inv)
    for name, raw in (("ori", raw_ori), ("inv", raw_inv)):
        k = keys3(raw["b"], raw["l"], raw["e"], L, E)
        if agg_mode == 1:
            uk, uv, arg = coalesce_max_with_arg(k, raw["v"], raw["edge"])
            out[name] = (uk, uv)
            out[name + "_arg"] = arg
        else:
            out[name] = coalesce_sum(k, raw["v"])
    out["ind"] = coalesce_sum(keys3(sp_b, sp_l, sp_e, L, E), ind_v)
    return out


def lookup(keys_table, vals_table, query):
    """Values of ``query`` keys in a sorted key table (0 where absent)."""
    query = np.asarray(query, np.int64)
    out = np.zeros(query.shape[0], F32)
    if keys_table.shape[0] == 0 or query.shape[0] == 0:
        return out
    pos = np.searchsorted(keys_table, query)
    safe = np.minimum(pos, keys_table.shape[0] - 1)
    hit = (pos < keys_table.shape[0]) & (keys_table[safe] == query)
    out[hit] = vals_table[safe[hit]]
    return out


def _edge_grad_factor(edge, edge_weight, is_score, scale):
    ew = np.asarray(edge_weight, F32).reshape(-1)[edge]
    if is_score:
        return (F32(1.0) / np.maximum(ew, F32(1e-12))).astype(F32)
    s = sigmoid_f32(ew * F32(scale))
    return (F32(scale) * (F32(1.0) - s)).astype(F32)


def sparse3d_backward(fwd, grads, sp_b, sp_l, sp_e, sp_v, w, B, L, E, r_size, wot_i=False,
                      agg_mode=0, edge_weight=None, is_score=False, scale=1.0,
                      want_edge_grad=False, num_facts=0):
    """Backward of one hop.  ``grads`` maps ori/inv/ind to coalesced (keys, vals).

    Sum mode: every raw message receives the gradient at its output key
    (fastlog.cu:2551-2606, fastlog_kernel.py:242-261).  Max mode: only the argmax
    message of each output key does (fastlog_kernel.py:153-167, fastlog.cu:2646-2676).
    Identity channel per fastlog.cu:2608-2644.  Edge-score gradient per
    fastlog_kernel.py:1032-1098.  Returns (grad_sp_value, grad_w, grad_edge or None).
    """
    sp_b = np.asarray(sp_b, np.int64); sp_l = np.asarray(sp_l, np.int64)
    sp_e = np.asarray(sp_e, np.int64); sp_v = np.asarray(sp_v, F32)
    w = np.asarray(w, F32)
    n = w.shape[2]
    grad_sp = np.zeros(sp_v.shape[0], F32)
    grad_w = np.zeros(w.shape, F32)
    gw_flat = grad_w.reshape(-1)
    grad_edge = np.zeros(num_facts, F32) if want_edge_grad else None
    for name, off in (("ori", 0), ("inv", r_size)):
        raw = fwd["raw_" + name]
        gk, gv = grads[name]
        if agg_mode == 1:
            okeys = fwd[name][0]
            arg = fwd[name + "_arg"]
            g = np.zeros(raw["v"].shape[0], F32)
            if okeys.shape[0] and gk.shape[0]:
                pos = np.searchsorted(okeys, gk)
                safe = np.minimum(pos, okeys.shape[0] - 1)
                ok = (pos < okeys.shape[0]) & (okeys[safe] == gk)
                g[arg[safe[ok]]] = gv[ok]
        else:
            g = lookup(gk, gv, keys3(raw["b"], raw["l"], raw["e"], L, E))
        if raw["v"].shape[0] == 0:
            continue
        ent = raw["entry"]
        ch = off + raw["rel"].astype(np.int64)
        wv = w[sp_b[ent], sp_l[ent], ch]
        gm = (g * raw["m"]).astype(F32)
        np.add.at(grad_sp, ent, (gm * wv).astype(F32))
        np.add.at(gw_flat, (sp_b[ent] * L + sp_l[ent]) * n + ch, (gm * sp_v[ent]).astype(F32))
        if want_edge_grad:
            fac = _edge_grad_factor(raw["edge"], edge_weight, is_score, scale)
            contrib = ((((g * sp_v[ent]).astype(F32) * wv).astype(F32) * raw["m"]).astype(F32) * fac).astype(F32)
            np.add.at(grad_edge, raw["edge"], contrib)
    if not wot_i:
        gk, gv = grads["ind"]
        g = lookup(gk, gv, keys3(sp_b, sp_l, sp_e, L, E))
        wid = w[sp_b, sp_l, n - 1]
        np.add.at(gw_flat, (sp_b * L + sp_l) * n + (n - 1), (g * sp_v).astype(F32))
        grad_sp += (g * wid).astype(F32)
    return grad_sp, grad_w, grad_edge


# ----------------------------------------------------------------------------
# bridge / proof-loop reducers
# ----------------------------------------------------------------------------

def sum_sparse3d_concat(*states):
    """Union-sum of coalesced states (fastlog_bridge.py:26-42)."""
    non_empty = [s for s in states if s[0].shape[0] > 0]
    if not non_empty:
        return np.empty(0, np.int64), np.empty(0, F32)
    if len(non_empty) == 1:
        return non_empty[0]
    return coalesce_sum(np.concatenate([s[0] for s in non_empty]),
                        np.concatenate([s[1] for s in non_empty]))


def sum_sp_3d(state, L, E):
    """Sum over rules → [B, E] keys ``b*E + e`` (fastlog_bridge.py:17-23)."""
    k, v = state
    b, _, e = split3(k, L, E)
    return coalesce_sum(b * E + e, v)


def _row_ids(keys, L, E):
    b, l, _ = split3(keys, L, E)
    return b * L + l


def normalize_sparse3d(state, B, L, E, eps=0.0, availability="mass"):
    """drum.py:31-51: drop zeros, divide each (b, l) row by its sum, optionally times
    ``min(sum, 1)``, drop zeros again."""
    k, v = state
    keep = v != 0
    k, v = k[keep], v[keep]
    rows = _row_ids(k, L, E)
    denom = np.zeros(B * L, F32)
    np.add.at(denom, rows, v)
    if eps > 0:
        denom = np.maximum(denom, F32(eps))
    out = (v / denom[rows]).astype(F32)
    if availability == "mass":
        out = (out * np.minimum(denom, F32(1.0))[rows]).astype(F32)
    elif availability != "none":
        raise ValueError(availability)
    keep = out != 0
    return k[keep], out[keep]


def norm_sp_3d(state, B, L, E):
    """src/model_mmDRUM_kernel_sp.py:39-52: row sums clamped at 1e-7, no mass factor."""
    k, v = state
    rows = _row_ids(k, L, E)
    denom = np.zeros(B * L, F32)
    np.add.at(denom, rows, v)
    denom = np.maximum(denom, F32(1e-7))
    out = (v / denom[rows]).astype(F32)
    keep = out != 0
    return k[keep], out[keep]


def prune_sparse3d_active_entities(state, E, topk_nodes):
    """drum.py:54-80.  Entity score = sum of |value| over (b, l).  ``torch.topk`` leaves
    the tie order unspecified; here ties keep the lower entity id."""
    k, v = state
    if topk_nodes <= 0 or v.shape[0] <= topk_nodes:
        return state
    kk = min(int(topk_nodes), int(E))
    ent = k % E
    score = np.zeros(E, F32)
    np.add.at(score, ent, np.abs(v))
    order = np.lexsort((np.arange(E), -score.astype(np.float64)))
    keep_ent = np.zeros(E, dtype=bool)
    keep_ent[order[:kk]] = True
    keep = keep_ent[ent]
    if keep.all():
        return state
    return k[keep], v[keep]


def _max_over_slots(keys2, slots, vals):
    """Max per ``keys2`` with ties to the smallest slot (sort key ``keys2*S + slot``)."""
    if keys2.shape[0] == 0:
        return np.empty(0, np.int64), np.empty(0, F32), np.empty(0, np.int64)
    order = np.lexsort((slots, -vals.astype(np.float64), keys2))
    sk = keys2[order]
    first = np.ones(sk.shape[0], dtype=bool)
    first[1:] = sk[1:] != sk[:-1]
    win = order[first]
    return keys2[win], vals[win], win


def max_sp_3d(state, L, E):
    """Max over rules per (b, e); ties → lowest rule index; zeros dropped
    (src/model_mmDRUM_kernel_sp.py:184-211)."""
    k, v = state
    b, l, e = split3(k, L, E)
    uk, uv, _ = _max_over_slots(b * E + e, l, v)
    keep = uv != 0
    return uk[keep], uv[keep]


def sparse3d_max(states, L, E):
    """Key-wise max across states; ties → earliest state in argument order; zeros dropped
    (src/model_mmDRUM_kernel_sp.py:237-270).  Returns (keys, vals, state index)."""
    ks = np.concatenate([s[0] for s in states]) if states else np.empty(0, np.int64)
    vs = np.concatenate([s[1] for s in states]) if states else np.empty(0, F32)
    sid = np.concatenate([np.full(s[0].shape[0], i, np.int64) for i, s in enumerate(states)]) \
        if states else np.empty(0, np.int64)
    uk, uv, win = _max_over_slots(ks, sid, vs)
    keep = uv != 0
    return uk[keep], uv[keep], sid[win][keep]


def norm_sp_3d_max(state, B, L, E):
    """src/model_mmDRUM_kernel_sp.py:165-181 (no dropout): normalise, then max over rules."""
    return max_sp_3d(norm_sp_3d(state, B, L, E), L, E)


def bound_scores(vals):
    """``1 - exp(-max(x, 0))`` in float32 (proof.py:642-649): the exponential is rounded
    to float32 first (from float64), then subtracted from 1 in float32, as the reference's
    float32 tensor arithmetic does."""
    x = np.maximum(np.asarray(vals, F32), F32(0.0))
    e = np.exp(-x.astype(np.float64)).astype(F32)
    return (F32(1.0) - e).astype(F32)


def ordered_tail_scores(tails, scores, cap=0):
    """Score descending, then tail ascending (decode_core.py:350-363)."""
    tails = np.asarray(tails, np.int64)
    scores = np.asarray(scores, F32)
    if tails.shape[0] == 0:
        return tails[:0], scores[:0]
    order = np.lexsort((tails, -scores))
    if cap > 0:
        order = order[:cap]
    return tails[order], scores[order]


def candidate_rows(keys2, vals, E):
    """proof.py:729-758: per query row the (tails, scores) arrays in key order."""
    rows = np.asarray(keys2, np.int64) // E
    tails = np.asarray(keys2, np.int64) % E
    out = {}
    if rows.shape[0] == 0:
        return out
    uniq, start = np.unique(rows, return_index=True)
    ends = np.concatenate([start[1:], [rows.shape[0]]])
    for r, s, e in zip(uniq.tolist(), start.tolist(), ends.tolist()):
        out[int(r)] = (tails[s:e], vals[s:e])
    return out


# ----------------------------------------------------------------------------
# the hop loop  (proof.py:467-614)  and the max-aggregation decode
# ----------------------------------------------------------------------------

def initial_state(heads, B, L, E):
    b = np.repeat(np.arange(B, dtype=np.int64), L)
    l = np.tile(np.arange(L, dtype=np.int64), B)
    e = np.repeat(np.asarray(heads, np.int64), L)
    return keys3(b, l, e, L, E), np.ones(B * L, F32)


def apply_threshold(state, threshold):
    if threshold <= 0:
        return state
    k, v = state
    keep = v >= F32(np.float32(threshold))
    return k[keep], v[keep]


def proof_sum_forward(heads, w_hops, csr, mask, edge_weight, B, L, E, R, cap=UNCAPPED,
                      topk_nodes=0, is_score=True, scale=1.0, threshold=0.0):
    """``kernel_sparse_scores`` (proof.py:467-614) with dropout off.

    Returns (final [B,E] (keys2, vals), trace) where trace holds, per hop, the input
    state, the op outputs and the concatenated / normalised states for the backward.
    """
    state = initial_state(heads, B, L, E)
    trace = []
    for hop in range(w_hops.shape[0]):
        state = prune_sparse3d_active_entities(state, E, topk_nodes)
        b, l, e = split3(state[0], L, E)
        fwd = sparse3d_forward(b, l, e, state[1], w_hops[hop], csr, mask, edge_weight, B, L, E, R,
                               wot_i=False, cap=cap, agg_mode=0, is_score=is_score, scale=scale)
        cat = sum_sparse3d_concat(fwd["ori"], fwd["inv"], fwd["ind"])
        nxt = normalize_sparse3d(cat, B, L, E, 0.0, "mass")
        nxt = apply_threshold(nxt, threshold)
        trace.append(dict(state=state, fwd=fwd, cat=cat, out=nxt))
        state = nxt
    return sum_sp_3d(state, L, E), trace


def _normalize_mass_backward(cat, out, g_out, B, L, E):
    """Gradient of ``normalize_sparse3d(.., 0, "mass")`` w.r.t. the concat values.

    x = (y / d) * min(d, 1), d = Σ_row y; clamp_max passes the gradient when d <= 1.
    """
    k, y = cat
    keep_in = y != 0
    gy = np.zeros(y.shape[0], F32)
    kk, yy = k[keep_in], y[keep_in]
    rows = _row_ids(kk, L, E)
    d = np.zeros(B * L, F32)
    np.add.at(d, rows, yy)
    c = np.minimum(d, F32(1.0))
    gx = lookup(out[0], g_out, kk)  # gradient only where the output kept the key
    q = (yy / d[rows]).astype(F32)
    g_q = (gx * c[rows]).astype(F32)
    g_c = np.zeros(B * L, F32)
    np.add.at(g_c, rows, (gx * q).astype(F32))
    g_d = np.zeros(B * L, F32)
    np.add.at(g_d, rows, (-(g_q * yy).astype(F32) / (d[rows] * d[rows])).astype(F32))
    g_d = (g_d + np.where(d <= 1.0, g_c, F32(0.0))).astype(F32)
    gyy = ((g_q / d[rows]).astype(F32) + g_d[rows]).astype(F32)
    gy[keep_in] = gyy
    return gy


def proof_sum_backward(trace, final_grad, w_hops, csr, mask, edge_weight, B, L, E, R,
                       is_score=True, scale=1.0, num_facts=0):
    """Gradients of the hop loop w.r.t. the per-hop rule weights and the edge scores.

    ``final_grad`` = (keys2, vals) on the final [B, E] output keys.
    Returns (grad_w_hops [hops,B,L,n], grad_edge [T]).
    """
    hops = len(trace)
    grad_w = np.zeros(w_hops.shape, F32)
    grad_edge = np.zeros(num_facts, F32)
    last = trace[-1]["out"]
    b, _, e = split3(last[0], L, E)
    g_state = lookup(final_grad[0], final_grad[1], b * E + e)  # d final / d last state
    for hop in range(hops - 1, -1, -1):
        tr = trace[hop]
        g_cat = _normalize_mass_backward(tr["cat"], tr["out"], g_state, B, L, E)
        ck = tr["cat"][0]
        fwd = tr["fwd"]
        grads = {name: (fwd[name][0], lookup(ck, g_cat, fwd[name][0])) for name in ("ori", "inv", "ind")}
        st = tr["state"]
        sb, sl, se = split3(st[0], L, E)
        gsp, gw, ge = sparse3d_backward(fwd, grads, sb, sl, se, st[1], w_hops[hop], B, L, E, R,
                                        agg_mode=0, edge_weight=edge_weight, is_score=is_score,
                                        scale=scale, want_edge_grad=True, num_facts=num_facts)
        grad_w[hop] = gw
        grad_edge += ge
        if hop > 0:
            prev_out = trace[hop - 1]["out"]
            g_state = lookup(st[0], gsp, prev_out[0])
    return grad_w, grad_edge


def proof_max_forward(heads, w_hops, csr, mask, edge_weight, B, L, E, R, cap=UNCAPPED,
                      is_score=True, scale=1.0):
    """Max-aggregation hop loop (src/model_mmDRUM_kernel_sp.py:388-445 with
    ``transition_reduce == "max"``): per hop the op with ``agg_mode=1``, then
    ``sparse3d_max(ind, ori, inv)``; ``norm_sp_3d`` between hops and ``norm_sp_3d_max``
    after the last.  Returns ([B,E] (keys2, vals), trace)."""
    state = initial_state(heads, B, L, E)
    hops = w_hops.shape[0]
    trace = []
    final = None
    for hop in range(hops):
        b, l, e = split3(state[0], L, E)
        fwd = sparse3d_forward(b, l, e, state[1], w_hops[hop], csr, mask, edge_weight, B, L, E, R,
                               wot_i=False, cap=cap, agg_mode=1, is_score=is_score, scale=scale)
        mk, mv, msid = sparse3d_max([fwd["ind"], fwd["ori"], fwd["inv"]], L, E)
        trace.append(dict(state=state, fwd=fwd, max=(mk, mv, msid)))
        if hop < hops - 1:
            state = norm_sp_3d((mk, mv), B, L, E)
        else:
            final = norm_sp_3d_max((mk, mv), B, L, E)
    return final, trace


def decode_topk(final, B, E, k):
    """Per query: bound the raw scores, order (score desc, tail asc), keep ``k``.

    Returns (tails int64 [B, k] padded with -1, scores f32 [B, k] padded with 0,
    counts int64 [B])."""
    keys2, vals = final
    scores = bound_scores(vals)
    rows = candidate_rows(keys2, scores, E)
    tails_out = np.full((B, k), -1, np.int64)
    scores_out = np.zeros((B, k), F32)
    counts = np.zeros(B, np.int64)
    for r, (t, s) in rows.items():
        ot, os_ = ordered_tail_scores(t, s, k)
        tails_out[r, :ot.shape[0]] = ot
        scores_out[r, :ot.shape[0]] = os_
        counts[r] = ot.shape[0]
    return tails_out, scores_out, counts


def count_messages(state, csr, w, L, E, R, cap=UNCAPPED):
    """Messages of one hop = Σ over frontier entries of the taken ori + inv edges."""
    b, l, e = split3(state[0], L, E)
    total = 0
    for off, base in ((0, 8), (R, 12)):
        _, _, take, _ = group_takes(b, l, e, np.asarray(w, F32), csr[base], csr[base + 1], csr[base + 3],
                                    off, cap)
        total += int(take.sum())
    return total


# ----------------------------------------------------------------------------
# query planning (decode_core.py:287-348, tnb_batching.py:12-20)
# ----------------------------------------------------------------------------

def tnb_batch_plan(dataset: str, nominal_batch_size: int):
    """(true_target_batch_size, false_main_batch_count) (tnb_batching.py:12-20)."""
    nominal = max(1, int(nominal_batch_size))
    false_count = 0 if dataset == "family" else min(nominal - 1, int(round(nominal * 0.5)))
    return max(1, nominal - false_count), false_count


def rule_first_hop_channels(logits, tau, threshold):
    """Channels c with max_l softmax(logits[0, l, :] / tau)[c] >= threshold (decode_core.py:302-307).

    ``logits`` [K, L, n] float32 for one relation; the softmax is taken in float64 and
    rounded to float32 (the reference's float32 softmax agrees to an ulp)."""
    z = np.asarray(logits[0], np.float64) / np.float64(np.float32(tau))
    z = z - z.max(axis=-1, keepdims=True)
    w = np.exp(z)
    w = (w / w.sum(axis=-1, keepdims=True)).astype(np.float32)
    return np.nonzero(w.max(axis=0) >= np.float32(threshold))[0].astype(np.int64)


def rule_first_hop_cache(head, rel, tail, supply, wanted, R):
    """channel -> sorted unique endpoints of the supplied facts (decode_core.py:308-331):
    heads of relation c under channel c, tails under channel c + R, for each wanted c."""
    head, rel, tail = (np.asarray(a, np.int64) for a in (head, rel, tail))
    supply = np.asarray(supply, bool)
    cache = {}
    for c in sorted(set(int(x) for x in wanted)):
        sel = supply & (rel == c)
        cache[c] = np.unique(head[sel])
        cache[c + R] = np.unique(tail[sel])
    return cache


def rule_first_hop_query_heads(channels, cache, query_heads):
    """Query heads (in order, duplicates kept) in the union of the channels' sets
    (decode_core.py:334-347); [] when no channel has a set."""
    sets = [cache[int(c)] for c in channels if int(c) in cache]
    if not sets:
        return np.zeros(0, np.int64)
    q = np.asarray(query_heads, np.int64)
    return q[np.isin(q, np.concatenate(sets))]


# ----------------------------------------------------------------------------
# decode accumulator: best-k cut per query row (decode.py:45-116)
# ----------------------------------------------------------------------------

def oracle_best_k(not_base, in_true, base_true):
    """The cut k in [0, n] of one ordered candidate row that maximises (base true + new true)
    - new wrong; ties: more true, then fewer wrong, then the smaller k (decode.py:45-69).
    Returns (k, wrong at k)."""
    nb = np.asarray(not_base, bool)
    nt = nb & np.asarray(in_true, bool)
    pn = np.concatenate([[0], np.cumsum(nb, dtype=np.int64)])
    pt = np.concatenate([[0], np.cumsum(nt, dtype=np.int64)])
    true_count = int(base_true) + pt
    wrong = pn - pt
    gain = true_count - wrong
    j = int(np.lexsort((np.arange(gain.shape[0]), wrong, -true_count, -gain))[0])
    return j, int(wrong[j])


class RelationAccumulator:
    """Counters of decode.py:72-116 (``_OracleRelationAccumulator``) restated."""

    def __init__(self):
        self.candidate_total = self.max_candidate_count = self.query_count = 0
        self.selected = self.selected_wrong = self.new = self.new_true = 0

    def add_row(self, ordered_tails, true_tails, base_tails) -> int:
        t = np.asarray(ordered_tails, np.int64)
        true = np.asarray(true_tails, np.int64)
        base = np.asarray(base_tails, np.int64)
        n = t.shape[0]
        self.candidate_total += n
        self.max_candidate_count = max(self.max_candidate_count, n)
        not_base = ~np.isin(t, base)
        in_true = np.isin(t, true)
        first = np.zeros(n, bool)
        if n:
            first[np.unique(t, return_index=True)[1]] = True
        new_unit = first & not_base
        cn = np.concatenate([[0], np.cumsum(new_unit, dtype=np.int64)])
        cnt = np.concatenate([[0], np.cumsum(new_unit & in_true, dtype=np.int64)])
        if n == 0 or true.shape[0] == 0:
            k, wrong = 0, 0
        else:
            k, wrong = oracle_best_k(not_base, in_true, int(np.isin(base, true).sum()))
        self.query_count += int(k > 0)
        self.selected += k
        self.selected_wrong += wrong
        self.new += int(cn[k])
        self.new_true += int(cnt[k])
        return k

    def counters(self):
        return [self.candidate_total, self.max_candidate_count, self.query_count, self.selected,
                self.selected_wrong, self.new, self.new_true]


# ----------------------------------------------------------------- rule-weight producer
# SupplyGatedDRUM._shared_rule_logits / build_rule_logits (drum.py:429-467) and the per-hop
# softmax of proof.py:569-571, per query row as the reference computes them, in float64.
# ``params``: emb [n, H]; lstm: list over rules of dicts with w_ih, w_hh [2, 4H, H] and
# b_ih, b_hh [2, 4H] (direction 0 = forward, 1 = reverse; torch.nn.LSTM gate rows i, f, g, o);
# w_lin [n, 2H], b_lin [n].

def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _lstm_direction(xs, w_ih, w_hh, b, reverse):
    """One LSTM direction over xs [S, B, H] (torch.nn.LSTM, drum.py:305): per step the
    activated gates (i, f, g, o), c and h, indexed by time."""
    S, B, H = xs.shape
    h = np.zeros((B, H))
    c = np.zeros((B, H))
    gates, cs, hs = [None] * S, [None] * S, [None] * S
    for t in (range(S - 1, -1, -1) if reverse else range(S)):
        pre = xs[t] @ w_ih.T + h @ w_hh.T + b
        i, f, g, o = _sigmoid(pre[:, :H]), _sigmoid(pre[:, H:2 * H]), np.tanh(pre[:, 2 * H:3 * H]), \
            _sigmoid(pre[:, 3 * H:])
        c = f * c + i * g
        h = o * np.tanh(c)
        gates[t], cs[t], hs[t] = (i, f, g, o), c, h
    return gates, cs, hs


def shared_rule_logits(params, rels, K):
    """logits [B, K, L, n] of drum.py:429-438 (sequence [emb[rel]] * K + [emb[-1]]) and the
    trace the backward needs."""
    emb = np.asarray(params["emb"], np.float64)
    rels = np.asarray(rels, np.int64)
    B = rels.size
    xs = np.stack([emb[rels]] * K + [np.broadcast_to(emb[-1], (B, emb.shape[1]))])  # [K+1, B, H]
    w_lin = np.asarray(params["w_lin"], np.float64)
    b_lin = np.asarray(params["b_lin"], np.float64)
    out, trace = [], []
    for lp in params["lstm"]:
        dirs = []
        for d in range(2):
            b = np.asarray(lp["b_ih"][d], np.float64) + np.asarray(lp["b_hh"][d], np.float64)
            dirs.append(_lstm_direction(xs, np.asarray(lp["w_ih"][d], np.float64),
                                        np.asarray(lp["w_hh"][d], np.float64), b, reverse=d == 1))
        o = np.concatenate([np.stack(dirs[0][2]), np.stack(dirs[1][2])], axis=-1)  # [K+1, B, 2H]
        out.append(o[:K].transpose(1, 0, 2) @ w_lin.T + b_lin)                     # [B, K, n]
        trace.append((dirs, o))
    return np.stack(out, axis=2), (xs, trace)


def invert_rule_logits(logits, R):
    """tclm_invert_rule_logits (drum.py:238-243)."""
    sw = np.concatenate([logits[..., R:2 * R], logits[..., :R], logits[..., 2 * R:]], axis=-1)
    return sw[:, ::-1]


def rule_softmax(logits, tau):
    """w [K, B, L, n] = softmax(logits[:, hop] / tau) per hop (proof.py:571)."""
    z = np.asarray(logits, np.float64) / tau
    z = z - z.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return (e / e.sum(axis=-1, keepdims=True)).transpose(1, 0, 2, 3)


def rule_softmax_backward(w, grad_w, tau):
    """d loss / d logits [B, K, L, n] from w, grad_w [K, B, L, n]."""
    g = w * (grad_w - (w * grad_w).sum(axis=-1, keepdims=True)) / tau
    return g.transpose(1, 0, 2, 3)


def shared_rule_logits_backward(params, rels, K, trace, grad_logits):
    """Gradients of shared_rule_logits for grad_logits [B, K, L, n] (BPTT of each direction):
    dict of emb, w_lin, b_lin and per rule w_ih, w_hh, b (= grad of b_ih = grad of b_hh)."""
    xs, rule_traces = trace
    emb = np.asarray(params["emb"], np.float64)
    w_lin = np.asarray(params["w_lin"], np.float64)
    rels = np.asarray(rels, np.int64)
    S, B, H = xs.shape
    g_emb = np.zeros_like(emb)
    g_wlin = np.zeros_like(w_lin)
    g_blin = np.zeros(w_lin.shape[0])
    rules = []
    for l, (lp, (dirs, o)) in enumerate(zip(params["lstm"], rule_traces)):
        gl = grad_logits[:, :, l, :].transpose(1, 0, 2)            # [K, B, n]
        g_wlin += np.einsum("tbn,tbk->nk", gl, o[:K])
        g_blin += gl.sum(axis=(0, 1))
        g_o = np.zeros((S, B, 2 * H))
        g_o[:K] = gl @ w_lin
        per_dir = {"w_ih": [], "w_hh": [], "b": []}
        g_x = np.zeros_like(xs)
        for d in range(2):
            gates, cs, hs = dirs[d]
            w_ih = np.asarray(lp["w_ih"][d], np.float64)
            w_hh = np.asarray(lp["w_hh"][d], np.float64)
            order = list(range(S - 1, -1, -1)) if d == 1 else list(range(S))
            gw_ih, gw_hh, gb = np.zeros_like(w_ih), np.zeros_like(w_hh), np.zeros(4 * H)
            dh_next = np.zeros((B, H))
            dc_next = np.zeros((B, H))
            for s in range(S - 1, -1, -1):
                t = order[s]
                i, f, g, o_ = gates[t]
                c = cs[t]
                c_prev = cs[order[s - 1]] if s > 0 else np.zeros((B, H))
                h_prev = hs[order[s - 1]] if s > 0 else np.zeros((B, H))
                dh = dh_next + g_o[t, :, d * H:(d + 1) * H]
                tc = np.tanh(c)
                dc = dc_next + dh * o_ * (1 - tc * tc)
                dpre = np.concatenate([dc * g * i * (1 - i), dc * c_prev * f * (1 - f), dc * i * (1 - g * g),
                                       dh * tc * o_ * (1 - o_)], axis=1)
                dc_next = dc * f
                dh_next = dpre @ w_hh
                g_x[t] += dpre @ w_ih
                gw_ih += dpre.T @ xs[t]
                gw_hh += dpre.T @ h_prev
                gb += dpre.sum(axis=0)
            per_dir["w_ih"].append(gw_ih)
            per_dir["w_hh"].append(gw_hh)
            per_dir["b"].append(gb)
        np.add.at(g_emb, rels, g_x[:K].sum(axis=0))
        g_emb[-1] += g_x[K].sum(axis=0)
        rules.append({k: np.stack(v) for k, v in per_dir.items()})
    return {"emb": g_emb, "w_lin": g_wlin, "b_lin": g_blin, "lstm": rules}


def build_rule_logits(params, rels, K, R, penalty=0.0, invert=False, table_index=None, table=None):
    """SupplyGatedDRUM.build_rule_logits (drum.py:440-467): the shared logits, or the target
    table's rows where a relation has one (all mapped: the table alone), the same-relation
    channel penalty, then the TCLM inversion.  Returns (logits [B, K, L, n], backward), where
    backward(grad_logits) -> the gradient dict of shared_rule_logits_backward plus "table"."""
    rels = np.asarray(rels, np.int64)
    B = rels.size
    trace, row, mapped = None, None, None
    if table_index is not None:
        row = np.asarray(table_index)[rels]
        mapped = row >= 0
        if mapped.all():
            logits = np.asarray(table, np.float64)[row]
        else:
            logits, trace = shared_rule_logits(params, rels, K)
            logits = logits.copy()
            logits[mapped] = np.asarray(table, np.float64)[row[mapped]]
    else:
        logits, trace = shared_rule_logits(params, rels, K)
    if penalty > 0:
        logits = logits.copy()
        rows = np.arange(B)
        logits[rows, :, :, rels] -= penalty
        logits[rows, :, :, rels + R] -= penalty
    if invert:
        logits = invert_rule_logits(logits, R)

    def backward(grad_logits):
        g = np.asarray(grad_logits, np.float64)
        if invert:
            g = invert_rule_logits(g, R)  # an involution
        grads = {}
        if table_index is not None:
            gt = np.zeros(np.asarray(table).shape)
            np.add.at(gt, row[mapped], g[mapped])
            grads["table"] = gt
            if trace is None:
                return grads
            g = g.copy()
            g[mapped] = 0.0
        grads.update(shared_rule_logits_backward(params, rels, K, trace, g))
        return grads

    return logits, backward
