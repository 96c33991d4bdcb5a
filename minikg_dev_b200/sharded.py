"""Destination-partitioned hop loop over several GPUs (one process per GPU, ``torch.distributed``).

The reference runs on one GPU.  For graphs whose ``B x L x E`` key space outgrows one device,
rank k owns the entities ``[lo_k, hi_k)`` (ranges balanced by how many messages can reach them)
and keeps the whole CSR pair resident (both directions, so per-entry edge caps are decided on
complete rows).  Per hop:

1. the sparse frontier is all-gathered: sizes first, then one padded payload of
   ``(key, value)`` per rank (``key = (b * L + l) * E + e``);
2. the per-hop op (``MergedHop``: ori, inv and ind reduced into one store, i.e. the concat-sum)
   expands every gathered entry but produces only messages whose destination rank k owns,
   into a key space of ``B x L x (hi_k - lo_k)``; outputs of different ranks are disjoint, so
   no reduction of messages is needed;
3. the mass normalisation (drum.py:31-50) divides by per-(b, l) column sums that are
   all-reduced; the optional state threshold is local;
4. what remains is rank k's part of the next frontier.

After the last hop the per-query sum over rules (proof.py:609) is local, and top-k decoding
merges per-rank candidates (score descending, then tail ascending, decode_core.py:350-363).
``topk_nodes`` pruning (drum.py:54-80) selects the global top entities from per-rank top
candidates, with equal scores ordered by entity id.

Gradients: the gather's backward all-reduces the frontier gradient and hands each rank the
slice of its own entries; the normalisation's written-out backward all-reduces its row sums
(``_NormalizeMass``); inputs replicated on every
rank (rule weights, edge scores) pass through ``replicated`` whose backward all-reduces, so
every rank ends with the full gradient of the sum of all ranks' local results.  Every rank
issues the same collectives in the same order, including for empty local frontiers.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist
from torch import autograd


# ----------------------------------------------------------------------------- partition
def plan_dst_ranges(message_in: torch.Tensor, world: int) -> list[int]:
    """Boundaries ``[0 = lo_0, ..., lo_world = E]`` balancing ``sum(message_in + 1)`` per range.

    ``message_in[e]`` is the number of facts that can deliver a message to ``e`` (its total
    degree over both directions); the +1 spreads entities without edges.  Every range is
    non-empty (``world <= E`` required)."""
    E = int(message_in.numel())
    if world < 1 or world > E:
        raise ValueError(f"cannot split {E} entities over {world} ranks")
    cum = torch.cumsum(message_in.detach().to("cpu", torch.int64) + 1, 0)
    total = int(cum[-1])
    bounds = [0]
    for k in range(1, world):
        target = (total * k) // world
        cut = int(torch.searchsorted(cum, torch.tensor(target, dtype=torch.int64), right=True))
        cut = max(cut, bounds[-1] + 1)           # non-empty range k-1
        cut = min(cut, E - (world - k))          # leave one entity for each remaining range
        bounds.append(cut)
    bounds.append(E)
    return bounds


def message_in_counts(head: torch.Tensor, tail: torch.Tensor, num_entities: int) -> torch.Tensor:
    """Facts that can deliver a message to each entity: ori messages go to the tail, inv
    messages to the head."""
    return (torch.bincount(tail.long(), minlength=num_entities) +
            torch.bincount(head.long(), minlength=num_entities))


# ----------------------------------------------------------------------------- collectives with autograd
class _Replicated(autograd.Function):
    """Identity forward; the backward all-reduces the gradient (a tensor every rank holds)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


def replicated(x: torch.Tensor, group=None) -> torch.Tensor:
    return _Replicated.apply(x, group)


class _Select(autograd.Function):
    """``v[sel]`` for unique positions ``sel``; the backward writes the gradient back without
    the accumulating index-put a general gather would need."""

    @staticmethod
    def forward(ctx, v, sel):
        ctx.save_for_backward(sel)
        ctx.n = int(v.numel())
        return v[sel]

    @staticmethod
    def backward(ctx, g):
        sel, = ctx.saved_tensors
        out = torch.zeros(ctx.n, dtype=g.dtype, device=g.device)
        out[sel] = g
        return out, None


def _all_gather_padded(t: torch.Tensor, counts: list[int], group) -> list[torch.Tensor]:
    """All-gathers the first dimension of ``t`` (this rank's ``counts[rank]`` rows) from every rank."""
    world = len(counts)
    m = max(max(counts), 1)
    pad = torch.zeros((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    return [bufs[r][: counts[r]] for r in range(world)]


def _gather_counts(n: int, device, group) -> list[int]:
    """Every rank's size; an impossible size (negative) raises the same error on all ranks,
    after the exchange, so no rank is left waiting in a later collective."""
    world = dist.get_world_size(group)
    c = torch.tensor([n], dtype=torch.int64, device=device)
    out = [torch.empty_like(c) for _ in range(world)]
    dist.all_gather(out, c, group=group)
    counts = [int(x) for x in torch.cat(out).tolist()]
    bad = [r for r, x in enumerate(counts) if x < 0]
    if bad:
        raise RuntimeError(f"sharded hop: rank(s) {bad} reported an invalid frontier size {[counts[r] for r in bad]}")
    return counts


def _frontier_size(keys: torch.Tensor) -> int:
    return int(keys.numel())


class _GatherFrontier(autograd.Function):
    """All ranks' ``(keys, values)`` concatenated in rank order.  Backward: the gradient of every
    gathered value is summed over ranks; each rank keeps the slice of its own entries."""

    @staticmethod
    def forward(ctx, keys, vals, group):
        counts = _gather_counts(_frontier_size(keys), keys.device, group)
        k_all = torch.cat(_all_gather_padded(keys, counts, group))
        v_all = torch.cat(_all_gather_padded(vals.detach(), counts, group))
        ctx.counts, ctx.group = counts, group
        ctx.rank = dist.get_rank(group)
        ctx.mark_non_differentiable(k_all)
        return k_all, v_all

    @staticmethod
    def backward(ctx, _gk, gv):
        counts, world = ctx.counts, len(ctx.counts)
        m = max(max(counts), 1)
        pad = torch.zeros((world, m), dtype=gv.dtype, device=gv.device)
        off = 0
        for r, c in enumerate(counts):
            pad[r, :c] = gv[off: off + c]
            off += c
        dist.all_reduce(pad, group=ctx.group)
        return None, pad[ctx.rank, : counts[ctx.rank]].clone(), None


class _NormalizeMass(autograd.Function):
    """normalize_sparse3d(.., 0, "mass") (drum.py:31-50) on this rank's key-sorted entries with
    the per-(b, l) row sums all-reduced over ranks, then the optional state threshold:
    ``x = (y / d) * min(d, 1)`` for y != 0; returns the kept positions (non-differentiable)
    and their values.  The backward is written out -- ``dy = dx * c / d + g_d[row]`` with
    ``g_d = sum_row(-dx * c * y / d^2) + [d <= 1] * sum_row(dx * y / d)``, the row sums again
    all-reduced -- so no gather / index-put backward of torch runs on the entries."""

    @staticmethod
    def forward(ctx, y, rows, nrows: int, threshold: float, group):
        yd = y.detach()
        d = torch.zeros(nrows, dtype=torch.float64, device=yd.device).index_add_(0, rows, yd.double())
        dist.all_reduce(d, group=group)
        d = d.to(yd.dtype)  # fp64 sums, rounded once
        dr = d[rows]
        c = d.clamp_max(1.0)
        nz = yd != 0
        x = torch.where(nz, yd / dr * c[rows], torch.zeros_like(yd))
        keep = x != 0
        if threshold > 0:
            keep &= x >= threshold
        sel = torch.nonzero(keep, as_tuple=True)[0]
        ctx.save_for_backward(yd, rows, d, sel)
        ctx.group, ctx.nrows, ctx.n = group, nrows, int(yd.numel())
        ctx.mark_non_differentiable(sel)
        return sel, x[sel]

    @staticmethod
    def backward(ctx, _g_sel, gx_sel):
        y, rows, d, sel = ctx.saved_tensors
        gx = torch.zeros(ctx.n, dtype=gx_sel.dtype, device=gx_sel.device)
        gx[sel] = gx_sel  # unique positions: no accumulation needed
        nz = y != 0
        dr = d[rows]
        c = d.clamp_max(1.0)
        q = torch.where(nz, y / dr, torch.zeros_like(y))
        g_q = gx * c[rows]
        zero = torch.zeros_like(y)
        part = torch.zeros((2, ctx.nrows), dtype=torch.float64, device=y.device)  # sums that cancel: fp64
        part[0].index_add_(0, rows, torch.where(nz, gx * q, zero).double())
        part[1].index_add_(0, rows, torch.where(nz, -(g_q * y) / (dr * dr), zero).double())
        dist.all_reduce(part, group=ctx.group)
        g_d = part[1] + torch.where(d <= 1.0, part[0], torch.zeros_like(part[0]))
        gy = torch.where(nz, (g_q.double() / dr.double() + g_d[rows]).to(y.dtype), zero)
        return gy, None, None, None, None


# ----------------------------------------------------------------------------- the loop
@dataclass
class ShardSpec:
    rank: int
    world: int
    bounds: list[int]          # world + 1 entity boundaries
    group: object = None

    @property
    def lo(self) -> int:
        return self.bounds[self.rank]

    @property
    def hi(self) -> int:
        return self.bounds[self.rank + 1]


# hop_fn(frontier keys, frontier values, w_h [B, L, n], lo, hi) -> (keys, values): the sum of
# the op's ori, inv and ind outputs whose destinations lie in [lo, hi), keys ascending
HopFn = Callable[..., tuple]


def cuda_hop_fn(graph, mask, edge_scores, cap: int, is_score: bool, scale: float) -> HopFn:
    """The per-hop op of this package on the resident ``DeviceGraph``: ``MergedHop`` (ori, inv
    and ind reduced into one key-sorted output) restricted to the rank's destinations."""
    from .sparse_loop import MergedHop

    def hop(keys, vals, w_h, lo, hi):
        return MergedHop.apply(keys, vals, w_h, edge_scores, graph, mask, bool(is_score), float(scale), int(cap),
                               int(lo), int(hi))
    return hop


def _coalesce_sum(keys: torch.Tensor, vals: torch.Tensor):
    uk, inv = torch.unique(keys, sorted=True, return_inverse=True)
    out = torch.zeros(uk.shape[0], dtype=vals.dtype, device=vals.device).index_add(0, inv, vals)
    return uk, out


def _prune_global(keys, vals, E: int, topk_nodes: int, spec: ShardSpec):
    """drum.py:54-80 across ranks: unless the whole state has at most ``topk_nodes`` entries,
    only the global top-``topk_nodes`` entities by summed |value| survive, ranked over all E
    entities with equal scores (zeros included) ordered by entity id.  A rank's top
    ``topk_nodes`` of its own range contains every global winner it owns, so per-rank
    candidates suffice.  Every rank issues the same collectives whatever its local size."""
    dev = vals.device
    total = torch.tensor([keys.numel()], dtype=torch.int64, device=dev)
    dist.all_reduce(total, group=spec.group)
    if int(total) <= topk_nodes:
        return keys, vals
    lo, hi = spec.lo, spec.hi
    ent = keys % E
    score = torch.zeros(hi - lo, dtype=vals.dtype, device=dev).index_add(0, ent - lo, vals.detach().abs())
    k = min(int(topk_nodes), E)
    order = torch.sort(score, descending=True, stable=True).indices[:k]
    counts = _gather_counts(int(order.numel()), dev, spec.group)
    ids = torch.cat(_all_gather_padded(order + lo, counts, spec.group))
    scs = torch.cat(_all_gather_padded(score[order], counts, spec.group))
    o1 = torch.sort(ids, stable=True).indices
    o2 = torch.sort(scs[o1], descending=True, stable=True).indices
    keep_ids = ids[o1][o2][:k]
    keep_ent = torch.zeros(hi - lo, dtype=torch.bool, device=dev)
    keep_ent[keep_ids[(keep_ids >= lo) & (keep_ids < hi)] - lo] = True
    sel = torch.nonzero(keep_ent[ent - lo], as_tuple=True)[0]
    return keys[sel], _Select.apply(vals, sel)


def message_counter(graph, cap: int):
    """Messages a gathered frontier sends: per entry min(out-degree, cap) per direction (the
    256-bucket cap takes exactly ``cap`` edges of a longer row)."""
    c = graph.csr
    deg = [(c[0][1:] - c[0][:-1]).long(), (c[4][1:] - c[4][:-1]).long()]
    cap = int(cap)

    def count(e_all):
        return sum(torch.clamp(d[e_all], max=cap).sum() for d in deg)
    return count


def sharded_proof_scores(spec: ShardSpec, hop_fn: HopFn, heads: torch.Tensor, w_hops: torch.Tensor, E: int,
                         threshold: float = 0.0, topk_nodes: int = 0, msg_counter=None, msgs_out=None):
    """``kernel_sparse_scores`` (proof.py:467-614, sum path, no dropout) with entities split
    over ranks.  ``w_hops`` [K, B, L, n] is replicated on every rank.  Returns this rank's
    part of the sparse [B, E] result as ``(keys b * E + e, values)`` (sorted keys, entities in
    ``[lo, hi)``).  With ``msg_counter`` (see ``message_counter``) the global message count of
    every hop is appended to ``msgs_out`` as a device scalar."""
    K, B, L, _ = (int(s) for s in w_hops.shape)
    dev = w_hops.device
    lo, hi = spec.lo, spec.hi
    w_rep = replicated(w_hops, spec.group)
    hd = heads.to(device=dev, dtype=torch.int64)
    b0 = torch.arange(B, device=dev).repeat_interleave(L)
    l0 = torch.arange(L, device=dev).repeat(B)
    e0 = hd.repeat_interleave(L)
    mine = (e0 >= lo) & (e0 < hi)
    keys = torch.sort(((b0 * L + l0) * E + e0)[mine]).values
    vals = torch.ones(keys.numel(), dtype=torch.float32, device=dev)
    for h in range(K):
        if topk_nodes > 0:
            keys, vals = _prune_global(keys, vals, E, topk_nodes, spec)
        k_all, v_all = _GatherFrontier.apply(keys, vals, spec.group)
        if msg_counter is not None:
            msgs_out.append(msg_counter(k_all % E))
        # the op's (ori + inv + ind) for this rank's destinations, coalesced in key order
        keys, y = hop_fn(k_all, v_all, w_rep[h], lo, hi)
        # normalize_sparse3d(.., 0, "mass") with global column sums, then the threshold
        sel, vals = _NormalizeMass.apply(y, keys // E, B * L, float(threshold), spec.group)
        keys = keys[sel]
    # sum_sp_3d: sum over rules
    be, e = keys // E, keys % E
    return _coalesce_sum((be // L) * E + e, vals)


def merge_topk(spec: ShardSpec, keys: torch.Tensor, vals: torch.Tensor, B: int, E: int, k: int):
    """Per query the top-``k`` (tail, bounded score) over all ranks, ordered by score descending
    then tail ascending (proof.py:642-649, 729-758; decode_core.py:350-363).  ``keys`` are
    ``b * E + e`` of this rank's raw scores.  Returns (tails [B, k] -1 padded, scores [B, k],
    counts [B]) on every rank."""
    dev = vals.device
    # bound 1 - exp(-max(x, 0)): exp in float64 rounded to float32, then the float32 difference
    sc = 1.0 - torch.exp(-vals.detach().clamp_min(0.0).double()).float()
    b, t = keys // E, keys % E
    # local top-k per query: order (b asc, score desc, tail asc), keep the first k of each b
    o = torch.sort(t, stable=True).indices
    o = o[torch.sort(sc[o], descending=True, stable=True).indices]
    o = o[torch.sort(b[o], stable=True).indices]
    bs = b[o]
    first = torch.searchsorted(bs, bs, right=False)
    rank_in_b = torch.arange(bs.numel(), device=dev) - first
    sel = o[rank_in_b < k]
    counts = _gather_counts(int(sel.numel()), dev, spec.group)
    gb = torch.cat(_all_gather_padded(b[sel], counts, spec.group))
    gt = torch.cat(_all_gather_padded(t[sel], counts, spec.group))
    gs = torch.cat(_all_gather_padded(sc[sel], counts, spec.group))
    o = torch.sort(gt, stable=True).indices
    o = o[torch.sort(gs[o], descending=True, stable=True).indices]
    o = o[torch.sort(gb[o], stable=True).indices]
    bs = gb[o]
    first = torch.searchsorted(bs, bs, right=False)
    pos = torch.arange(bs.numel(), device=dev) - first
    take = pos < k
    tails = torch.full((B, k), -1, dtype=torch.int64, device=dev)
    scores = torch.zeros((B, k), dtype=torch.float32, device=dev)
    tails[bs[take], pos[take]] = gt[o][take]
    scores[bs[take], pos[take]] = gs[o][take].to(torch.float32)
    cnt = torch.bincount(bs[take], minlength=B)
    return tails, scores, cnt
