"""The sum hop loop on sparse states, fused around the per-hop op.

``SparseHopLoop`` computes what the reference's hop loop composes from the op and the bridge
reducers (proof.py:569-609: ``prune_sparse3d_active_entities`` -> op ->
``sum_sparse3d_concat`` -> ``normalize_sparse3d(.., 0, "mass")``, then ``sum_sp_3d``) for any
edge cap, with the state kept as sorted ``(key, value)`` arrays (``key = (b * L + l) * E + e``):

* the op runs with ``merge_outputs``: ori, inv and ind messages are reduced into one store
  (dense key slab or hash table, chosen from the exact message count), so the concat-sum
  costs nothing and comes out coalesced in key order;
* the mass normalisation divides by per-(b, l) row sums (rows are contiguous in key order);
* the backward is written out: the normalisation's gradient
  ``dy = dx * c / d + sum_row(-dx * c * y / d^2) + [d <= 1] * sum_row(dx * y / d)``
  (c = min(d, 1)), then the op's backward with that one gradient store serving ori, inv and
  ind, then the prune mask.

No torch sparse coalesce or index-put backward runs.  The hop-by-hop torch composition
(``proof.sparse_hop_loop``) stays for dropout during training.
"""
from __future__ import annotations

import ctypes

import torch
from torch import autograd

from . import _native as N
from . import fastlog_kernel as FK
from .graph import DeviceGraph
from .slab_loop import _mass_normalize, _mass_normalize_grad
from .sparse_reducers import _reduce


class _HopState:
    __slots__ = ("keys_in", "vals_in", "prune_sel", "idx_y", "keys_y", "y", "d", "keep", "params", "n_pre")


def _frontier_arrays(keys: torch.Tensor, L: int, E: int):
    be = keys // E
    return (be // L).contiguous(), (be % L).contiguous(), (keys % E).contiguous()


def _prune(keys, vals, E: int, topk_nodes: int):
    """drum.py:54-80 on sorted keys: the top-``topk_nodes`` entities by summed |value| over the
    whole batch survive (equal scores: lower entity id), unless the state has at most
    ``topk_nodes`` entries.  Returns (keys, vals, selected positions or None)."""
    if topk_nodes <= 0 or keys.numel() <= topk_nodes:
        return keys, vals, None
    ent = keys % E
    score = torch.zeros(E, dtype=vals.dtype, device=vals.device).index_add_(0, ent, vals.detach().abs())
    order = torch.sort(score, descending=True, stable=True).indices[: min(int(topk_nodes), E)]
    keep_ent = torch.zeros(E, dtype=torch.bool, device=vals.device)
    keep_ent[order] = True
    sel = torch.nonzero(keep_ent[ent], as_tuple=True)[0]
    if sel.numel() == keys.numel():
        return keys, vals, None
    return keys[sel], vals[sel], sel


def _op_forward(g: DeviceGraph, keys, vals, w_h, factor, B, L, cap, keep_alive, lo: int = 0, hi: int = 0):
    """The merged op (destinations in [lo, hi) when hi > lo): returns (indices [3, U], keys [U],
    values [U], params, message count)."""
    lib = N.load()
    dev = vals.device
    E = g.num_entities
    b, l, e = _frontier_arrays(keys, L, E)
    v = vals.detach().to(torch.float32).contiguous()
    keep_alive += [b, l, e, v]
    fr = N.Frontier(b.data_ptr(), l.data_ptr(), e.data_ptr(), v.data_ptr(), int(keys.numel()))
    n = int(w_h.shape[-1])
    params = [B, L, E, g.num_relations, n, 0, 0, int(cap), int(lo), int(hi), 0, FK.ACCUM_MODES[FK.ACCUM], 1]
    p = N.HopParams(*params)
    st = N.stream_handle(dev)
    mc = torch.empty(2, dtype=torch.int64, device=dev)
    N.check(lib.mkg_hop_count_messages(ctypes.byref(g.struct), ctypes.byref(fr), ctypes.byref(p), mc.data_ptr(),
                                       N.error_word(dev).data_ptr(), st), "hop_count_messages")
    m_ori, m_inv = (int(x) for x in mc.tolist())
    if FK.ACCUM != "dense":
        params[10] = max(1, m_ori + m_inv + int(keys.numel()))  # the merged store holds all three
        p = N.HopParams(*params)
    nnz = int(keys.numel())
    ws = N.workspace(lib.mkg_hop_forward_workspace_bytes(ctypes.byref(p), nnz), dev)
    counts = torch.zeros(3, dtype=torch.int64, device=dev)
    N.check(lib.mkg_hop_forward(ctypes.byref(g.struct), ctypes.byref(fr), w_h.data_ptr(), ctypes.byref(factor),
                                ctypes.byref(p), ws.data_ptr(), ws.numel(), counts.data_ptr(),
                                N.error_word(dev).data_ptr(), st), "hop_forward")
    U = int(counts[0].item())
    N.raise_device_errors(dev)
    idx = torch.empty((3, U), dtype=torch.int64, device=dev)
    y = torch.empty(U, dtype=torch.float32, device=dev)
    N.check(lib.mkg_hop_emit(ctypes.byref(p), nnz, ws.data_ptr(), ws.numel(), 0, U, idx.data_ptr(), y.data_ptr(),
                             None, st), "hop_emit")
    keys_y = (idx[0] * L + idx[1]) * E + idx[2]
    return idx, keys_y, y, tuple(params), m_ori + m_inv


def _op_backward(g: DeviceGraph, st: _HopState, w_h, factor, gy, want_edge: bool):
    lib = N.load()
    dev = gy.device
    B, L = st.params[0], st.params[1]
    E = g.num_entities
    keep = []
    b, l, e = _frontier_arrays(st.keys_in, L, E)
    v = st.vals_in.detach().to(torch.float32).contiguous()
    keep += [b, l, e, v]
    fr = N.Frontier(b.data_ptr(), l.data_ptr(), e.data_ptr(), v.data_ptr(), int(st.keys_in.numel()))
    p = N.HopParams(*st.params)
    gv = gy.to(torch.float32).contiguous()
    keep.append(gv)
    go = N.Coo3(st.idx_y.data_ptr(), gv.data_ptr(), int(gv.numel()))
    empty = N.Coo3(None, None, 0)
    grad_sp = torch.empty(int(st.keys_in.numel()), dtype=torch.float32, device=dev)
    grad_w = torch.empty(tuple(w_h.shape), dtype=torch.float32, device=dev)
    grad_edge = torch.empty(g.num_facts, dtype=torch.float32, device=dev) if want_edge else None
    ws = N.workspace(lib.mkg_hop_backward_workspace_bytes(ctypes.byref(p), int(st.keys_in.numel())), dev)
    N.check(lib.mkg_hop_backward(ctypes.byref(g.struct), ctypes.byref(fr), w_h.data_ptr(), ctypes.byref(factor),
                                 ctypes.byref(p), ctypes.byref(go), ctypes.byref(empty), ctypes.byref(empty),
                                 None, None, None, None, None, None, None, grad_sp.data_ptr(), grad_w.data_ptr(),
                                 N.ptr(grad_edge), ws.data_ptr(), ws.numel(), N.error_word(dev).data_ptr(),
                                 N.stream_handle(dev)), "hop_backward")
    return grad_sp, grad_w, grad_edge


class MergedHop(autograd.Function):
    """One hop with ori, inv and ind reduced into one output (``sum_sparse3d_concat`` of the
    three), restricted to destinations in [lo, hi) when hi > lo: ``(keys, values)`` with keys
    ``(b * L + l) * E + e`` in ascending order.  Gradients for the frontier values, ``w`` and
    the edge scores.  The frontier keys need not be sorted."""

    @staticmethod
    def forward(ctx, keys, vals, w_h, edge_scores, graph: DeviceGraph, mask, is_score: bool, scale: float, cap: int,
                lo: int, hi: int):
        B, L = int(w_h.shape[0]), int(w_h.shape[1])
        keep_alive = []
        ew = edge_scores.detach().reshape(-1) if edge_scores is not None else None
        factor = N.edge_factor(mask, ew, bool(is_score), float(scale), keep_alive)
        wf = w_h.detach().to(torch.float32).contiguous()
        st = _HopState()
        st.keys_in, st.vals_in = keys, vals.detach()
        st.idx_y, st.keys_y, y, st.params, _ = _op_forward(graph, keys, vals, wf, factor, B, L, cap, keep_alive,
                                                           lo, hi)
        ctx.st, ctx.g, ctx.factor, ctx.keep_alive, ctx.wf = st, graph, factor, keep_alive, wf
        ctx.want_edge = edge_scores is not None and ctx.needs_input_grad[3]
        ctx.edge_shape = tuple(edge_scores.shape) if edge_scores is not None else None
        ctx.edge_dtype = edge_scores.dtype if edge_scores is not None else None
        ctx.mark_non_differentiable(st.keys_y)
        return st.keys_y, y

    @staticmethod
    def backward(ctx, _g_keys, gy):
        grad_sp, gw, ge = _op_backward(ctx.g, ctx.st, ctx.wf, ctx.factor, gy, ctx.want_edge)
        N.raise_device_errors(gy.device)
        ge = ge.view(ctx.edge_shape).to(ctx.edge_dtype) if ge is not None else None
        return None, grad_sp, gw, ge, None, None, None, None, None, None, None


class SparseHopLoop(autograd.Function):
    """``(w_hops [K, B, L, n], edge_scores [T]) -> (keys b * E + e, values, messages [K])`` of the
    sum hop loop on sparse states; gradients for ``w_hops`` and ``edge_scores``."""

    @staticmethod
    def forward(ctx, w_hops, edge_scores, heads, graph: DeviceGraph, mask, is_score: bool, scale: float, cap: int,
                topk_nodes: int, threshold: float):
        N.require_cuda(w_hops, "w_hops")
        K, B, L, n = (int(s) for s in w_hops.shape)
        g = graph
        E = g.num_entities
        if n != 2 * g.num_relations + 1:
            raise ValueError(f"w_hops has {n} channels, expected 2R+1 = {2 * g.num_relations + 1}")
        dev = g.device
        keep_alive = []
        wf = w_hops.detach().to(torch.float32).contiguous()
        ew = edge_scores.detach().reshape(-1) if edge_scores is not None else None
        factor = N.edge_factor(mask, ew, bool(is_score), float(scale), keep_alive)
        hd = heads.to(device=dev, dtype=torch.int64)
        keys = torch.sort((torch.arange(B * L, device=dev) * E + hd.repeat_interleave(L))).values
        vals = torch.ones(B * L, dtype=torch.float32, device=dev)
        hops, msgs = [], []
        for h in range(K):
            st = _HopState()
            st.n_pre = int(keys.numel())
            keys, vals, st.prune_sel = _prune(keys, vals, E, int(topk_nodes))
            st.keys_in, st.vals_in = keys, vals
            st.idx_y, st.keys_y, st.y, st.params, m = _op_forward(g, keys, vals, wf[h], factor, B, L, cap, keep_alive)
            msgs.append(m)
            d = N.row_sums(st.keys_y, st.y, E, B * L).to(torch.float32)  # fp64 sums in key order, rounded once
            x, dropped = _mass_normalize(st.keys_y, st.y, E, B * L, d, threshold)
            st.d, st.keep = d, None
            if dropped:  # zeros (explicit zero messages) or values under the threshold leave the state
                keep = x != 0
                if threshold > 0:
                    keep &= x >= threshold
                st.keep = keep
                keys, vals = st.keys_y[keep], x[keep]
            else:
                keys, vals = st.keys_y, x
            hops.append(st)
        # sum_sp_3d: the sum over rules, coalesced on the device (fp64 run sums)
        out_keys, out_vals, inv, _ = _reduce(((keys // E) // L) * E + keys % E, vals, 0)
        ctx.hops, ctx.inv, ctx.g = hops, inv, g
        ctx.factor, ctx.keep_alive = factor, keep_alive
        ctx.wf, ctx.shape = wf, (K, B, L, n)
        ctx.want_edge = edge_scores is not None and ctx.needs_input_grad[1]
        ctx.edge_shape = tuple(edge_scores.shape) if edge_scores is not None else None
        ctx.edge_dtype = edge_scores.dtype if edge_scores is not None else None
        ctx.mark_non_differentiable(out_keys)
        m_t = torch.tensor(msgs, dtype=torch.int64, device=dev)
        ctx.mark_non_differentiable(m_t)
        return out_keys, out_vals, m_t

    @staticmethod
    def backward(ctx, _g_keys, g_vals, _g_msgs):
        g = ctx.g
        E = g.num_entities
        K, B, L, n = ctx.shape
        dev = g_vals.device
        grad_w = torch.zeros(ctx.shape, dtype=torch.float32, device=dev)
        grad_edge = torch.zeros(g.num_facts, dtype=torch.float32, device=dev) if ctx.want_edge else None
        g_state = g_vals.to(torch.float32)[ctx.inv]
        for h in range(K - 1, -1, -1):
            st = ctx.hops[h]
            if st.keep is None:
                gx = g_state.to(torch.float32).contiguous()
            else:
                gx = torch.zeros_like(st.y)
                gx[st.keep] = g_state
            # the normalisation gradient: both row sums in one fp64 pass, then per entry
            gy = _mass_normalize_grad(st.keys_y, st.y, gx, E, B * L, st.d, None)
            grad_sp, gw, ge = _op_backward(g, st, ctx.wf[h], ctx.factor, gy, ctx.want_edge)
            grad_w[h] = gw
            if ge is not None:
                grad_edge += ge
            if st.prune_sel is not None:
                full = torch.zeros(st.n_pre, dtype=torch.float32, device=dev)
                full[st.prune_sel] = grad_sp
                grad_sp = full
            g_state = grad_sp
        N.raise_device_errors(dev)
        ge_out = grad_edge.view(ctx.edge_shape).to(ctx.edge_dtype) if grad_edge is not None else None
        return grad_w, ge_out, None, None, None, None, None, None, None, None


def sparse_proof_scores(graph: DeviceGraph, heads: torch.Tensor, w_hops: torch.Tensor,
                        edge_scores: torch.Tensor | None, mask: torch.Tensor | None = None, is_score: bool = True,
                        scale: float = 1.0, cap: int = 1 << 60, topk_nodes: int = 0,
                        threshold: float = 0.0, dense: bool = False):
    """The hop loop's result as a sparse ``[B, E]`` tensor (``dense=True``: dense) and the
    per-hop message counts."""
    K, B, L, n = (int(s) for s in w_hops.shape)
    E = graph.num_entities
    keys, vals, msgs = SparseHopLoop.apply(w_hops, edge_scores, heads, graph, mask, is_score, scale, int(cap),
                                           int(topk_nodes), float(threshold))
    out = torch.sparse_coo_tensor(torch.stack([keys // E, keys % E]), vals, (B, E), is_coalesced=True)
    return (out.to_dense() if dense else out), msgs
