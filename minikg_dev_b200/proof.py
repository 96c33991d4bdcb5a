"""The multi-hop proof engine: ``kernel_sparse_scores`` on the fused CUDA hop loop.

``HopLoopSum`` runs every hop of proof.py:467-614 (the op, ``sum_sparse3d_concat``,
``normalize_sparse3d(.., 0, "mass")``, then ``sum_sp_3d``) in one library call
(``mkg_proof_forward``) on a dense entity-major state, and its backward
(``mkg_proof_backward``) returns gradients for the per-hop rule weights and the edge
scores.  ``decode_max`` runs the max-aggregation loop (op with ``agg_mode=1`` →
``sparse3d_max(ind, ori, inv)`` → ``norm_sp_3d`` / ``norm_sp_3d_max``) and the decode
ordering (bound, score desc, tail asc, top-k) in ``mkg_proof_decode_max``.
``decode_max_sparse`` runs the same loop hop by hop on sparse states (any edge cap, graphs
whose dense state does not fit), with ``norm_sp_3d`` row sums added in key order
(``mkg_segment_sum_ordered``) so its result stays bit-exact too.

``kernel_sparse_scores(model, heads, rels, graph, args, is_training)`` keeps the
reference signature.  The fused loop covers uncapped hops and edge caps up to
DENSE_CAP_MAX (per-hop take tables of the capped rows, ``DeviceGraph.cap_index``) while the
dense state fits on the device; larger caps, entity pruning that is not a no-op, or graphs
too large for a dense state run the sparse loop (``sparse_loop.SparseHopLoop``), and dropout
while training runs hop by hop as the reference composes it.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native as N
from .fastlog_kernel import HopRange
from .graph import DeviceGraph, build_csr_structure
from .rules import rule_weights
from .sparse_reducers import (max_sp_3d, normalize_sparse3d, prune_sparse3d_active_entities, sparse3d_max, sum_sp_3d,
                              sum_sparse3d_concat)

UNCAPPED = 1 << 60
DENSE_CAP_MAX = 255  # MKG_DENSE_CAP_MAX: edge caps the fused loop takes


def dense_cap(topk_edges: int) -> int | None:
    """The fused loop's cap for the reference's ``topk_edges``: UNCAPPED, a cap in
    [0, DENSE_CAP_MAX] (a cap <= 0 takes no edge), or None (larger caps: the sparse loop)."""
    c = int(topk_edges)
    if c >= UNCAPPED:
        return UNCAPPED
    c = max(c, 0)
    return c if c <= DENSE_CAP_MAX else None


def _params(graph: DeviceGraph, B, L, hops, threshold=0.0, topk_edges=UNCAPPED):
    """Loop parameters; a capped loop carries the graph's cap index for ``topk_edges``."""
    cap = dense_cap(topk_edges)
    if cap is None:
        raise ValueError(f"the fused loop takes edge caps up to {DENSE_CAP_MAX} (got {topk_edges})")
    ix = graph.cap_index(cap) if cap < UNCAPPED else None
    p = N.ProofParams(int(B), int(L), graph.num_entities, graph.num_relations, int(hops), int(cap), float(threshold), 0,
                      None, None, ctypes.cast(ctypes.pointer(ix), ctypes.c_void_p) if ix is not None else None)
    return p, ix


class ProofRunner:
    """One hop-loop configuration on one graph with its workspace (reused across calls).

    ``forward`` keeps every hop's state in the workspace; ``backward`` consumes it, so a
    forward must precede each backward.  Optional ``torch.cuda.Event`` lists (2 per hop)
    are recorded around the pull kernels of each hop.
    """

    def __init__(self, graph: DeviceGraph, B: int, L: int, hops: int, threshold: float = 0.0,
                 topk_edges: int = UNCAPPED):
        lib = N.load()
        self.graph = graph
        self.B, self.L, self.K = int(B), int(L), int(hops)
        self.n = 2 * graph.num_relations + 1
        self.p, self._cap_ix = _params(graph, B, L, hops, threshold, topk_edges)
        self.ws = N.workspace(lib.mkg_proof_workspace_bytes(ctypes.byref(self.p)), graph.device)
        self._keep = []

    def _events(self, events):
        if events is None:
            return None
        arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        self._keep.append(arr)
        return ctypes.cast(arr, ctypes.c_void_p)

    def forward(self, heads, w_hops, out=None, msgs=None, events=None):
        lib = N.load()
        g = self.graph
        dev = g.device
        if tuple(w_hops.shape) != (self.K, self.B, self.L, self.n):
            raise ValueError(f"w_hops must be {(self.K, self.B, self.L, self.n)}, got {tuple(w_hops.shape)}")
        wf = w_hops.detach().to(torch.float32).contiguous()
        hd = heads.to(device=dev, dtype=torch.int64).contiguous()
        out = torch.empty((self.B, g.num_entities), dtype=torch.float32, device=dev) if out is None else out
        msgs = torch.zeros(self.K, dtype=torch.int64, device=dev) if msgs is None else msgs
        self._keep = [wf, hd]
        self.p.fwd_events, self.p.bwd_events = self._events(events), None
        adj = g.adjacency()
        N.check(lib.mkg_proof_forward(ctypes.byref(g.struct), ctypes.byref(adj), hd.data_ptr(), wf.data_ptr(),
                                      ctypes.byref(self.p), self.ws.data_ptr(), self.ws.numel(), out.data_ptr(),
                                      msgs.data_ptr(), N.error_word(dev).data_ptr(), N.stream_handle(dev)),
                "proof_forward")
        self.p.fwd_events = None
        return out, msgs

    def backward(self, grad_out, mask, edge_scores, is_score, scale, want_edge_grad: bool, grad_w=None,
                 grad_edge=None, events=None):
        lib = N.load()
        g = self.graph
        dev = g.device
        keep = []
        f = N.edge_factor(mask, edge_scores, is_score, scale, keep)
        go = grad_out.detach().to(torch.float32).contiguous()
        if grad_w is None:
            grad_w = torch.empty((self.K, self.B, self.L, self.n), dtype=torch.float32, device=dev)
        if want_edge_grad and grad_edge is None:
            grad_edge = torch.empty(g.num_facts, dtype=torch.float32, device=dev)
        self.p.bwd_events = self._events(events)
        adj = g.adjacency()
        N.check(lib.mkg_proof_backward(ctypes.byref(g.struct), ctypes.byref(adj), None, ctypes.byref(self.p),
                                       ctypes.byref(f), go.data_ptr(), grad_w.data_ptr(),
                                       N.ptr(grad_edge) if want_edge_grad else None, self.ws.data_ptr(),
                                       self.ws.numel(), N.error_word(dev).data_ptr(), N.stream_handle(dev)),
                "proof_backward")
        self.p.bwd_events = None
        return grad_w, (grad_edge if want_edge_grad else None)

    def capture(self, heads, w_hops, out, msgs, grad_out, edge_scores, grad_w, grad_edge=None, mask=None,
                is_score: bool = True, scale: float = 1.0, host_inputs=(), host_outputs=()) -> "torch.cuda.CUDAGraph":
        """One training step (edge-factor refresh, forward, backward) captured as a CUDA graph
        over these buffers.  Write new inputs into ``heads`` / ``w_hops`` / ``edge_scores`` /
        ``grad_out`` (and ``mask``) in place, then ``graph.replay()`` reruns the step with no
        host work; results land in ``out``, ``msgs``, ``grad_w``, ``grad_edge``.  The library
        does no host synchronisation inside a step, so the whole step is capturable.

        ``host_inputs``: (device tensor, pinned host tensor) pairs copied host to device at the
        start of every replay, so new inputs can be written into the host tensors instead;
        ``host_outputs``: (pinned host tensor, device tensor) pairs copied device to host at its
        end (read them after a synchronisation of the replaying stream)."""
        dev = self.graph.device
        for name, t, dt in (("heads", heads, torch.int64), ("w_hops", w_hops, torch.float32),
                            ("out", out, torch.float32), ("msgs", msgs, torch.int64),
                            ("grad_out", grad_out, torch.float32), ("edge_scores", edge_scores, torch.float32),
                            ("grad_w", grad_w, torch.float32)):
            if t.device != dev or t.dtype != dt or not t.is_contiguous():
                raise ValueError(f"capture: {name} must be a contiguous {dt} tensor on {dev}")
        host_inputs, host_outputs = list(host_inputs), list(host_outputs)
        for kind, pairs, d_at in (("host_inputs", host_inputs, 0), ("host_outputs", host_outputs, 1)):
            for pair in pairs:
                d, h = pair[d_at], pair[1 - d_at]
                if (d.device != dev or h.device.type != "cpu" or not h.is_pinned() or d.dtype != h.dtype
                        or d.shape != h.shape or not d.is_contiguous() or not h.is_contiguous()):
                    raise ValueError(f"capture: {kind} pairs a contiguous tensor on {dev} with a pinned "
                                     "host tensor of the same shape and dtype")
        want_edge = grad_edge is not None

        def step():
            for d, h in host_inputs:
                d.copy_(h, non_blocking=True)
            self.graph.set_edge_factor(mask, edge_scores, is_score, scale)
            self.forward(heads, w_hops, out, msgs)
            self.backward(grad_out, mask, edge_scores, is_score, scale, want_edge, grad_w, grad_edge)
            for h, d in host_outputs:
                h.copy_(d, non_blocking=True)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()  # warm-up outside the capture (lazy adjacency, kernel attributes)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        return graph

    def row_activity(self, hop: int) -> torch.Tensor:
        """uint8 [E]: entities holding a non-zero state value when hop ``hop`` starts."""
        lib = N.load()
        flags = torch.empty(self.graph.num_entities, dtype=torch.uint8, device=self.graph.device)
        N.check(lib.mkg_proof_row_activity(ctypes.byref(self.p), self.ws.data_ptr(), self.ws.numel(), int(hop),
                                           flags.data_ptr(), N.stream_handle(self.graph.device)), "row_activity")
        return flags


class HopLoopSum(torch.autograd.Function):
    """Sum-aggregation hop loop: ``(w_hops [K,B,L,n], edge_scores [T]) -> out [B,E]``."""

    @staticmethod
    def forward(ctx, w_hops, edge_scores, heads, graph: DeviceGraph, mask, is_score: bool, scale: float,
                threshold: float, topk_edges: int = UNCAPPED):
        K, B, L, n = (int(s) for s in w_hops.shape)
        if n != 2 * graph.num_relations + 1:
            raise ValueError(f"w_hops has {n} channels, expected 2R+1 = {2 * graph.num_relations + 1}")
        graph.set_edge_factor(mask, edge_scores, is_score, scale)
        runner = ProofRunner(graph, B, L, K, threshold, topk_edges)
        out, msgs = runner.forward(heads, w_hops)
        ctx.runner = runner
        ctx.mask, ctx.is_score, ctx.scale = mask, bool(is_score), float(scale)
        ctx.edge_scores = edge_scores.detach() if edge_scores is not None else None
        ctx.want_edge = edge_scores is not None and ctx.needs_input_grad[1]
        ctx.mark_non_differentiable(msgs)
        return out, msgs

    @staticmethod
    def backward(ctx, grad_out, _grad_msgs):
        runner: ProofRunner = ctx.runner
        # the factor column of the neighbour lists may have been rewritten by a later forward
        runner.graph.set_edge_factor(ctx.mask, ctx.edge_scores, ctx.is_score, ctx.scale)
        grad_w, grad_edge = runner.backward(grad_out, ctx.mask, ctx.edge_scores, ctx.is_score, ctx.scale,
                                            ctx.want_edge)
        ge = None
        if grad_edge is not None:
            ge = grad_edge.view(ctx.edge_scores.shape).to(ctx.edge_scores.dtype)
        return grad_w, ge, None, None, None, None, None, None, None


def proof_scores(graph: DeviceGraph, heads: torch.Tensor, w_hops: torch.Tensor, edge_scores: torch.Tensor | None,
                 mask: torch.Tensor | None = None, is_score: bool = True, scale: float = 1.0,
                 threshold: float = 0.0, topk_edges: int = UNCAPPED):
    """Dense raw scores ``[B, E]`` of the hop loop and the per-hop message counts ``[K]``;
    ``topk_edges`` <= DENSE_CAP_MAX caps every entry's messages as the reference's op does."""
    return HopLoopSum.apply(w_hops, edge_scores, heads, graph, mask, is_score, scale, threshold, topk_edges)


@dataclass
class DecodeResult:
    raw: torch.Tensor      # [B, E] raw max scores (0 = no proof)
    tails: torch.Tensor    # [B, k] int64, -1 padded
    scores: torch.Tensor   # [B, k] float32 bounded scores
    counts: torch.Tensor   # [B] int64


def decode_max(graph: DeviceGraph, heads: torch.Tensor, w_hops: torch.Tensor, topk: int,
               edge_scores: torch.Tensor | None, mask: torch.Tensor | None = None, is_score: bool = True,
               scale: float = 1.0, topk_edges: int = UNCAPPED) -> DecodeResult:
    """Max-aggregation hop loop + decode order (score desc, tail asc), top-``topk`` per query
    (``topk_edges`` <= DENSE_CAP_MAX: the reference's edge cap on every hop)."""
    lib = N.load()
    dev = graph.device
    K, B, L, n = (int(s) for s in w_hops.shape)
    E, R = graph.num_entities, graph.num_relations
    wf = w_hops.detach().to(torch.float32).contiguous()
    hd = heads.to(device=dev, dtype=torch.int64).contiguous()
    graph.set_edge_factor(mask, edge_scores, is_score, scale)
    p, _ix = _params(graph, B, L, K, 0.0, topk_edges)
    ws = N.workspace(lib.mkg_decode_workspace_bytes(ctypes.byref(p), int(topk)), dev)
    raw = torch.empty((B, E), dtype=torch.float32, device=dev)
    tails = torch.empty((B, int(topk)), dtype=torch.int64, device=dev)
    scores = torch.empty((B, int(topk)), dtype=torch.float32, device=dev)
    counts = torch.empty(B, dtype=torch.int64, device=dev)
    adj = graph.adjacency()
    N.check(lib.mkg_proof_decode_max(ctypes.byref(graph.struct), ctypes.byref(adj), hd.data_ptr(), wf.data_ptr(),
                                     ctypes.byref(p), int(topk), raw.data_ptr(), tails.data_ptr(),
                                     scores.data_ptr(), counts.data_ptr(), ws.data_ptr(), ws.numel(),
                                     N.error_word(dev).data_ptr(), N.stream_handle(dev)), "proof_decode_max")
    return DecodeResult(raw, tails, scores, counts)


def decode_topk(raw: torch.Tensor, topk: int):
    """bound_sparse_scores + sparse_candidate_rows + ordered_tail_scores on a dense [B, E]
    score matrix (entries != 0 are the candidates): (tails, scores, counts)."""
    lib = N.load()
    N.require_cuda(raw, "raw")
    r = raw.detach().to(torch.float32).contiguous()
    B, E = (int(s) for s in r.shape)
    tails = torch.empty((B, int(topk)), dtype=torch.int64, device=r.device)
    scores = torch.empty((B, int(topk)), dtype=torch.float32, device=r.device)
    counts = torch.empty(B, dtype=torch.int64, device=r.device)
    N.check(lib.mkg_decode_topk(r.data_ptr(), B, E, int(topk), tails.data_ptr(), scores.data_ptr(),
                                counts.data_ptr(), N.stream_handle(r.device)), "decode_topk")
    return tails, scores, counts


def norm_sp_3d_ordered(s: torch.Tensor) -> torch.Tensor:
    """norm_sp_3d (src/model_mmDRUM_kernel_sp.py:39-52) with each (b, l) row sum added in key
    order, as the reference's CPU index_put_ accumulates: value / clamp(row sum, 1e-7),
    zeros dropped."""
    s = s.coalesce()
    idx, val = s.indices(), s.values().to(torch.float32).contiguous()
    B, L, _ = s.shape
    rows = (idx[0] * L + idx[1]).contiguous()
    seg = torch.searchsorted(rows, torch.arange(B * L + 1, device=rows.device, dtype=rows.dtype))
    denom = N.segment_sum(seg, val, ordered=True)
    out = val / denom.clamp(min=1e-7)[rows]
    keep = out != 0
    return torch.sparse_coo_tensor(idx[:, keep], out[keep], s.shape, is_coalesced=True)


def sparse_topk(keys: torch.Tensor, vals: torch.Tensor, B: int, E: int, k: int):
    """Decode order on sparse raw scores (keys ``b * E + e``): bound ``1 - exp(-max(x, 0))``
    (exp rounded from double, then the fp32 difference), score descending, tail ascending,
    ``k`` per query (proof.py:642-649, 729-758; decode_core.py:350-363).  ``keys`` ascending.
    Returns (tails [B, k] -1 padded, scores [B, k], counts [B])."""
    dev = vals.device
    if 1 <= k <= 1024:  # one block per query: radix select + sort (mkg_sparse_topk)
        lib = N.load()
        N.require_cuda(vals, "vals")
        kc = keys.to(torch.int64).contiguous()
        vc = vals.detach().to(torch.float32).contiguous()
        tails = torch.empty((B, k), dtype=torch.int64, device=dev)
        scores = torch.empty((B, k), dtype=torch.float32, device=dev)
        counts = torch.empty(B, dtype=torch.int64, device=dev)
        ws = N.workspace(lib.mkg_sparse_topk_workspace_bytes(int(kc.numel())), dev)
        N.check(lib.mkg_sparse_topk(N.ptr(kc), N.ptr(vc), int(kc.numel()), int(B), int(E), int(k), tails.data_ptr(),
                                    scores.data_ptr(), counts.data_ptr(), ws.data_ptr(), ws.numel(),
                                    N.stream_handle(dev)), "sparse_topk")
        return tails, scores, counts
    # longer candidate lists: three stable sorts (tail, then score, then query)
    inside = (keys >= 0) & (keys < B * E)
    keys, vals = keys[inside], vals[inside]
    sc = 1.0 - torch.exp(-vals.detach().clamp_min(0.0).double()).float()
    b, t = keys // E, keys % E
    o = torch.sort(t, stable=True).indices
    o = o[torch.sort(sc[o], descending=True, stable=True).indices]
    o = o[torch.sort(b[o], stable=True).indices]
    bs = b[o]
    pos = torch.arange(bs.numel(), device=dev) - torch.searchsorted(bs, bs)
    take = pos < k
    tails = torch.full((B, k), -1, dtype=torch.int64, device=dev)
    scores = torch.zeros((B, k), dtype=torch.float32, device=dev)
    tails[bs[take], pos[take]] = t[o][take]
    scores[bs[take], pos[take]] = sc[o][take]
    return tails, scores, torch.bincount(bs[take], minlength=B)


@torch.no_grad()
def decode_max_sparse(graph: DeviceGraph, heads: torch.Tensor, w_hops: torch.Tensor, topk: int,
                      edge_scores: torch.Tensor | None, mask: torch.Tensor | None = None, cap: int = UNCAPPED,
                      is_score: bool = True, scale: float = 1.0):
    """The max-aggregation loop of src/model_mmDRUM_kernel_sp.py:388-445 hop by hop on sparse
    states (op with ``agg_mode=1`` and the edge cap -> ``sparse3d_max(ind, ori, inv)`` ->
    ``norm_sp_3d`` between hops, ``norm_sp_3d_max`` after the last), then ``sparse_topk``.
    Returns (final sparse [B, E] raw scores, tails, scores, counts)."""
    K, B, L, n = (int(x) for x in w_hops.shape)
    E = graph.num_entities
    dev = graph.device
    hd = heads.to(device=dev, dtype=torch.int64)
    state = torch.sparse_coo_tensor(
        torch.stack([torch.arange(B, device=dev).repeat_interleave(L), torch.arange(L, device=dev).repeat(B),
                     hd.repeat_interleave(L)]), torch.ones(B * L, device=dev), [B, L, E]).coalesce()
    mk = mask if mask is not None else torch.ones((), dtype=torch.float32, device=dev)
    wf = w_hops.to(device=dev, dtype=torch.float32)
    final = None
    for h in range(K):
        idx = state.indices()
        o, i, d = HopRange.apply(idx[0], idx[1], idx[2], state.values(), wf[h], graph, mk, edge_scores, B, L, False,
                                 int(cap), 1, bool(is_score), float(scale), 0, 0)
        s = sparse3d_max(d, o, i)
        if h < K - 1:
            state = norm_sp_3d_ordered(s)
        else:
            final = max_sp_3d(norm_sp_3d_ordered(s)).coalesce()
    fi = final.indices()
    keys = fi[0] * E + fi[1]
    tails, scores, counts = sparse_topk(keys, final.values(), B, E, int(topk))
    return final, tails, scores, counts


# ---------------------------------------------------------------------------- drop-in
def _device_graph_for(model, graph) -> DeviceGraph:
    """The model-level CSR cache of proof.py:496-506, holding a ``DeviceGraph``."""
    cache_key = (graph.e2triple[0].data_ptr(), graph.triple2e[1].data_ptr(), graph.r2triple[0].data_ptr())
    if getattr(model, "_b200_graph_key", None) != cache_key:
        csr = build_csr_structure(graph.e2triple[0], graph.triple2e[1], graph.r2triple[0], model.entity_count,
                                  model.relation_count)
        model._kernel_csr = csr
        model._b200_graph = DeviceGraph(csr, model.entity_count, model.relation_count)
        model._b200_graph_key = cache_key
    return model._b200_graph


FUSED_MAX_CHANNELS = (200 * 1024 // 4 - 128) // 128  # the backward stages dW [n, 128] in shared memory


def dense_state_fits(graph: DeviceGraph, B: int, L: int, hops: int, fraction: float = 0.5) -> bool:
    """Whether the fused loop takes this graph: at most FUSED_MAX_CHANNELS relation channels,
    and dense [E, B*L] states (every hop's, forward and backward) within ``fraction`` of the
    device's free memory.  Other graphs run the sparse loop."""
    if 2 * graph.num_relations + 1 > FUSED_MAX_CHANNELS:
        return False
    p = N.ProofParams(int(B), int(L), graph.num_entities, graph.num_relations, int(hops), UNCAPPED, 0.0, 0,
                      None, None, None)
    need = int(N.load().mkg_proof_workspace_bytes(ctypes.byref(p)))
    free, _total = torch.cuda.mem_get_info(graph.device)
    return need <= fraction * free


def _edge_inputs(model, graph, is_training):
    """Edge scores / mask exactly as proof.py:525-550 picks them (score path)."""
    edge_scores = model.weight
    if is_training and torch.is_grad_enabled():
        edge_scores = edge_scores.reshape(-1).clone()
    else:
        edge_scores = edge_scores.reshape(-1)
    mask = graph.mask_float if getattr(graph, "mask_float", None) is not None else None
    return edge_scores, mask, True, 1.0


def kernel_sparse_scores(model, heads, rels, graph, args, is_training: bool, dense: bool = False):
    """Drop-in for proof.py:467-614 (score edge-weight path).

    Returns the sparse ``[B, E]`` result of the reference (``dense=True``: the dense
    matrix, which the reference's consumers also accept).
    """
    g = _device_graph_for(model, graph)
    B, L, E, R, K = heads.shape[0], model.rules, model.entity_count, model.relation_count, model.step
    # rule weights of every hop, [K, B, L, n] (proof.py:524, 569-571): the LSTM producer and the
    # softmax on the device (rules.py)
    w_all = rule_weights(model, rels)
    edge_scores, mask, is_score, scale = _edge_inputs(model, graph, is_training)
    topk_edges = int(args.kernel_topk_edges)
    topk_nodes = int(args.kernel_topk_nodes)
    p_drop = float(getattr(getattr(model, "dropout", None), "p", 0.0) or 0.0)
    cap = dense_cap(topk_edges)
    fused = (cap is not None and (topk_nodes <= 0 or topk_nodes >= E) and not (is_training and p_drop > 0)
             and dense_state_fits(g, heads.shape[0], L, K))
    if fused:
        out, _ = HopLoopSum.apply(w_all, edge_scores, heads, g, mask, is_score, scale, 0.0, cap)
        return out if dense else out.to_sparse_coo().coalesce()
    if cap == UNCAPPED and not (is_training and p_drop > 0):
        # uncapped hops on a graph the dense state does not take: the key-slab loop
        from .slab_loop import slab_engine, slab_proof_scores
        out, _ = slab_proof_scores(slab_engine(g), heads, w_all, edge_scores, mask, is_score, scale, topk_nodes,
                                   0.0, dense=dense)
        return out
    if not (is_training and p_drop > 0):
        # larger caps, pruning or a graph too large for the dense state: the sparse loop fused
        # around the op (merged outputs, written-out backward)
        from .sparse_loop import sparse_proof_scores
        out, _ = sparse_proof_scores(g, heads, w_all, edge_scores, mask, is_score, scale, topk_edges,
                                     topk_nodes, 0.0, dense=dense)
        return out
    w_hops = [w_all[hop] for hop in range(K)]
    # dropout while training: hop by hop, as the reference composes it
    out = sparse_hop_loop(g, heads, w_hops, edge_scores, mask, is_score, scale, topk_edges, topk_nodes,
                          dropout=model.dropout)
    return out.to_dense() if dense else out


def sparse_hop_loop(g: DeviceGraph, heads: torch.Tensor, w_hops, edge_scores: torch.Tensor | None,
                    mask: torch.Tensor | None, is_score: bool = True, scale: float = 1.0, topk_edges: int = UNCAPPED,
                    topk_nodes: int = 0, dropout=None, msgs_out: list | None = None) -> torch.Tensor:
    """The sum hop loop of proof.py:569-609 on sparse states: per hop the prune, the op
    (``FastLogFunctionSparse3DTopK`` semantics: any cap, dense or hash message store),
    ``sum_sparse3d_concat`` and ``normalize_sparse3d(.., 0, "mass")`` (+ dropout when
    given), then ``sum_sp_3d``.  Differentiable in ``w_hops`` and ``edge_scores``.  With
    ``msgs_out`` the exact message count of every hop is appended (device scalars)."""
    B, L, _ = (int(x) for x in w_hops[0].shape)
    E, R = g.num_entities, g.num_relations
    dev = g.device
    state = torch.sparse_coo_tensor(
        torch.stack([torch.arange(B, device=dev).repeat_interleave(L), torch.arange(L, device=dev).repeat(B),
                     heads.to(dev).long().repeat_interleave(L)]),
        torch.ones(B * L, device=dev), [B, L, E]).coalesce()
    mvals = mask if mask is not None else torch.ones((), dtype=torch.float32, device=dev)
    if msgs_out is not None:
        c = g.csr
        deg = [(c[0][1:] - c[0][:-1]).long(), (c[4][1:] - c[4][:-1]).long()]
    for w_t in w_hops:
        state = prune_sparse3d_active_entities(state, topk_nodes)
        idx = state.indices()
        if msgs_out is not None:
            msgs_out.append(sum(torch.clamp(d_[idx[2]], max=max(int(topk_edges), 0)).sum() for d_ in deg))
        o, i, d = HopRange.apply(idx[0], idx[1], idx[2], state.values(), w_t, g, mvals, edge_scores, B, L, False,
                                 int(topk_edges), 0, bool(is_score), float(scale), 0, 0)
        state = normalize_sparse3d(sum_sparse3d_concat(o, i, d), 0.0, "mass")
        if dropout is not None:
            state = torch.sparse_coo_tensor(state.indices(), dropout(state.values()), state.shape).coalesce()
    return sum_sp_3d(state)
