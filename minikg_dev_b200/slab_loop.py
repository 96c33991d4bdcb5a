"""The uncapped sum hop loop on the key-slab engine (large graphs, sparse frontiers).

``kernel_sparse_scores`` (proof.py:467-614, sum path, dropout off) composes per hop the
``prune_sparse3d_active_entities`` prune (drum.py:54-80), the op (fastlog_kernel.py:900-984
with ``topk_edges`` uncapped), ``sum_sparse3d_concat`` (fastlog_bridge.py:26-42) and
``normalize_sparse3d(.., 0, "mass")`` (drum.py:31-51), then ``sum_sp_3d``
(fastlog_bridge.py:17-23).  ``SlabHopLoop`` runs that loop on the key-slab kernels of
``csrc/mkg_slab.cu``:

* a hop's messages (ori, inv and identity at once: the concat-sum) are added into a store
  with one fp32 slot per output key of a window of (b, l) rows and a touched bit per slot,
  entity-major (a destination's rows adjacent: the rules of one query share their frontier
  entities, so their messages land in the same sectors); the touched keys come out in
  entity-major order (ascending entity, then row) by a bitmap popcount scan, with fp64 row
  sums for the normalisation, and the store is left zeroed for the next use -- no sort, no
  hash table.  Frontiers stay in that order from hop to hop;
* the normalisation is elementwise on the emitted values; the final sum over rules is a
  reduce-by-key to the ``(b, e)`` keys (``mkg_reduce_by_key``: sorted output, and the inverse
  map that spreads the result's gradient back over the rules);
* the backward is written out: the normalisation gradient with fp64 row sums, then the
  transposed walk with the output gradient held in the store (fp64 entry and rule-weight
  accumulators), hop by hop down to the first.

With a ``ShardSpec`` the loop is destination-partitioned over ranks (one process per GPU):
rank k owns the entities ``[lo_k, hi_k)``, keeps only the push records whose destination it
owns (so every message is walked by exactly one rank), all-gathers the frontier each hop (the
ranks' entity-major lists, concatenated in rank order, are the whole frontier in entity-major
order) and all-reduces the normalisation's row sums; the backward all-reduces the frontier gradient, the
row sums of the normalisation gradient, and at the end the rule-weight and edge-score
gradients.  Every rank issues the same collectives in the same order.  With one process the
same code runs without collectives.
"""
from __future__ import annotations

import ctypes

import torch
from torch import autograd

from . import _native as N
from .graph import DeviceGraph

STORE_FRACTION = 0.45   # at most this share of the free device memory for the slab store
# destinations per tile (a tile's touched sectors stay in the 126 MB L2): measured on the
# 4.6 M-entity step, 1 / 2 / 4 / 8 tiles gave 10.94 / 10.34 / 10.04 / 10.49 ms
TILE_ENTITIES = 1_200_000


def _restrict(full_ptr, full_push, full_degree, lo: int, hi: int, E: int):
    """(ptr [E + 1] int32, records, positions in the full list) of the push records whose
    destination lies in [lo, hi)."""
    dev = full_push.device
    nbr = full_push[:, 0]
    sel = torch.nonzero((nbr >= lo) & (nbr < hi), as_tuple=True)[0]
    push = full_push[sel].contiguous()
    rows = torch.repeat_interleave(torch.arange(E, device=dev), full_degree)
    cnt = torch.bincount(rows[sel], minlength=E)
    ptr = torch.zeros(E + 1, dtype=torch.int32, device=dev)
    ptr[1:] = torch.cumsum(cnt, 0).to(torch.int32)
    return ptr, push, sel


class SlabEngine:
    """Resident state of the key-slab loop on one GPU: the push list (the graph's, or only the
    records whose destination lies in ``[lo, hi)``), cut into destination *tiles*, a zero-kept
    slab store and its window size.

    A tile is a sub-range of the destinations with its own push list (the records that reach
    it): a hop's expansion (and its backward walk) is one launch that walks the tiles in turn
    (up to ``SLAB_MAX_TILES`` per launch), so the updates in flight touch only one tile's part
    of the entity-major store, whose sectors then stay in L2 (a whole 4.6 M-entity range's
    touched sectors do not: every message then fetched and wrote back its sector); the
    collect, the gradient's put and the clearing run once over the whole window.
    ``dst_tiles`` (default: one per ``TILE_ENTITIES`` destinations) sets their number.

    ``store_bytes`` caps the store (default: ``STORE_FRACTION`` of the free memory when first
    sized); a window then covers as many (b, l) rows of the destination range as fit, and a hop
    whose rows exceed it runs window by window."""

    def __init__(self, graph: DeviceGraph, lo: int = 0, hi: int = 0, store_bytes: int | None = None,
                 dst_tiles: int | None = None):
        self.g = graph
        self.dev = graph.device
        E = graph.num_entities
        self.lo, self.hi = (int(lo), int(hi)) if hi > lo else (0, E)
        self.extent = self.hi - self.lo
        graph.adjacency()
        keep = graph._adj_keep
        self.full_ptr = keep["push_ptr"]
        self.full_push = keep["push"]
        self.full_degree = (self.full_ptr[1:] - self.full_ptr[:-1]).to(torch.int64)
        nt = int(dst_tiles) if dst_tiles else max(1, -(-self.extent // TILE_ENTITIES))
        nt = max(1, min(nt, self.extent))
        edges = [self.lo + (self.extent * t) // nt for t in range(nt + 1)]
        # tiles: (lo, extent, ptr, push); a single tile over the whole graph shares its lists
        self.tiles = []
        if nt == 1 and self.lo == 0 and self.hi == E:
            self.tiles.append((0, E, self.full_ptr, self.full_push))
            self.ptr, self._shared = self.full_ptr, True
        else:
            for t in range(nt):
                ptr_t, push_t, _ = _restrict(self.full_ptr, self.full_push, self.full_degree, edges[t], edges[t + 1], E)
                self.tiles.append((edges[t], edges[t + 1] - edges[t], ptr_t, push_t))
            # the engine's whole-range degrees (for byte accounting)
            self.ptr = torch.zeros(E + 1, dtype=torch.int32, device=self.dev)
            for _, _, ptr_t, _ in self.tiles:
                self.ptr += ptr_t
            self._shared = False
        # launch groups of at most SLAB_MAX_TILES tiles: (count, host arrays of the tiles' device
        # list pointers); each group's expansion is one launch walking its tiles in turn
        self.tile_groups = []
        for g0 in range(0, len(self.tiles), N.SLAB_MAX_TILES):
            grp = self.tiles[g0:g0 + N.SLAB_MAX_TILES]
            ptrs = (ctypes.c_void_p * len(grp))(*[p.data_ptr() for _, _, p, _ in grp])
            recs = (ctypes.c_void_p * len(grp))(*[r.data_ptr() for _, _, _, r in grp])
            self.tile_groups.append((len(grp), ptrs, recs))
        self._store_cap = store_bytes
        self._budget_bound = False
        self.store = None
        self.rows_per_window = 0
        # when a list: (kind, [(start, end) event per launch], algorithmic bytes, tiles) per hop
        # window, for roofline accounting (adds host synchronisations; off by default)
        self.trace = None
        self._groups = None

    @property
    def records(self) -> int:
        return sum(int(push.shape[0]) for _, _, _, push in self.tiles)

    def set_edge_factor(self, mask, weight, is_score: bool, scale: float) -> None:
        """Rewrites the factor field of this engine's push records from the mask / edge scores
        (tile lists: each holds copies of its records)."""
        if self._shared:
            self.g.set_edge_factor(mask, weight, is_score, scale, push_only=True)
            return
        keep = []
        f = N.edge_factor(mask, weight, is_score, scale, keep)
        for _, _, _, push in self.tiles:
            N.check(N.load().mkg_records_set_factor(push.data_ptr(), int(push.shape[0]), self.g.num_facts,
                                                    ctypes.byref(f), N.stream_handle(self.dev)),
                    "records_set_factor")
        self.g.factor_writes += 1

    def ensure_store(self, rows: int) -> None:
        """Sizes the zero-kept store: ``rows`` (b, l) rows of the destination range, or as many
        as the budget holds (then kept: the budget does not grow)."""
        lib = N.load()
        if self.store is not None and (self.rows_per_window >= rows or self._budget_bound):
            return
        budget = self._store_cap
        if budget is None:
            free, _ = torch.cuda.mem_get_info(self.dev)
            budget = int(STORE_FRACTION * (free + (self.store.numel() if self.store is not None else 0)))
        per_row = int(lib.mkg_slab_store_bytes(self.extent * 64)) / 64.0
        fit = max(1, min(int(rows), int(budget // per_row)))
        self._budget_bound = fit < rows
        self.store = None
        nbytes = int(lib.mkg_slab_store_bytes(fit * self.extent))
        self.store = torch.zeros(nbytes, dtype=torch.uint8, device=self.dev)
        self.rows_per_window = fit

    def window(self, row0: int, nrows: int) -> N.SlabWindow:
        return N.SlabWindow(self.g.num_entities, int(row0), int(nrows), self.lo, self.extent)


# ----------------------------------------------------------------------------- kernels, windowed
def _windows(total_rows: int, per: int):
    for r0 in range(0, total_rows, per):
        yield r0, min(per, total_rows - r0)


def entity_major(keys: torch.Tensor, vals: torch.Tensor, E: int, BL: int):
    """``(keys, vals)`` reordered to entity-major order (ascending entity, then row)."""
    if keys.numel() == 0:
        return keys, vals
    order = torch.sort((keys % E) * BL + keys // E).indices
    return keys[order], vals[order]


def _events(eng: SlabEngine):
    if eng.trace is None:
        return None
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    ev[0].record()
    return ev


def _in_rows(x, E: int, r0: int, nr: int, whole: bool):
    return x if whole else x[((x // E) >= r0) & ((x // E) < r0 + nr)]


def _collect(eng: SlabEngine, win, norm=None):
    """Emits the touched keys of the store (entity-major order) with their values; with ``norm``
    = (fp32 row sums of the window's rows, threshold) also their mass-normalised values and a
    device count of the results the loop drops (``mkg_slab_emit_normalized``)."""
    lib = N.load()
    dev = eng.dev
    st = N.stream_handle(dev)
    slots = win.nrows * win.extent
    ws = N.workspace(lib.mkg_slab_collect_workspace_bytes(slots), dev)
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    N.check(lib.mkg_slab_count(ctypes.byref(win), eng.store.data_ptr(), ws.data_ptr(), ws.numel(), cnt.data_ptr(),
                               st), "slab_count")
    U = int(cnt.item())
    keys = torch.empty(U, dtype=torch.int64, device=dev)
    vals = torch.empty(U, dtype=torch.float32, device=dev)
    if norm is None:
        N.check(lib.mkg_slab_emit(ctypes.byref(win), eng.store.data_ptr(), ws.data_ptr(), ws.numel(), U,
                                  keys.data_ptr(), vals.data_ptr(), st), "slab_emit")
        return keys, vals
    d32, threshold = norm
    x = torch.empty(U, dtype=torch.float32, device=dev)
    dropped = torch.zeros(1, dtype=torch.int64, device=dev)
    N.check(lib.mkg_slab_emit_normalized(ctypes.byref(win), eng.store.data_ptr(), ws.data_ptr(), ws.numel(), U,
                                         d32.data_ptr(), float(threshold), keys.data_ptr(), vals.data_ptr(),
                                         x.data_ptr(), dropped.data_ptr(), st), "slab_emit_normalized")
    return keys, vals, x, dropped


def graph_bytes(eng: SlabEngine, keys) -> int:
    """Compulsory graph bytes of a hop whose frontier holds ``keys``: per distinct source its
    records (4 B neighbour + 4 B edge score each), relation groups (10 B each: 2 B relation, 4 B
    start, 4 B count) and row pointers (8 B)."""
    if keys.numel() == 0:
        return 0
    E = eng.g.num_entities
    if eng._groups is None:
        c = eng.g.csr
        eng._groups = ((c[8][1:] - c[8][:-1]) + (c[12][1:] - c[12][:-1])).to(torch.int64)
    src = torch.unique(keys % E)
    deg = (eng.ptr[1:] - eng.ptr[:-1]).to(torch.int64)[src]
    grp = torch.where(deg > 0, eng._groups[src], torch.zeros_like(deg))
    return int((deg * 8 + grp * 10 + 8).sum())


def expand_forward(eng: SlabEngine, keys, vals, w_h, BL: int, check: bool = True, agg_mode: int = 0,
                   normalize=None):
    """One hop's concat-summed output over the engine's destinations: (keys in entity-major order
    within each row window, windows in row order; values; fp64 row sums [BL], zeros for
    ``agg_mode`` 1, which keeps each key's largest message instead; the output's [a, b) part of
    every row window, in window order).  The frontier may come in any order
    (entity-major keeps neighbouring atomics in the same sectors).  ``check``: refuse frontier
    keys outside [B, L, E] on the host (the loop, whose keys are its own outputs, skips that
    synchronisation).

    ``normalize`` = (ShardSpec or None, threshold), sum hop only: the hop's mass normalisation
    (drum.py:31-51) with the row sums all-reduced over ranks (one all-reduce per hop on every
    path); returns (keys, raw values, fp32 row sums [BL], parts, normalised values, number of
    them the loop drops).  With one row window the values are normalised as they are gathered
    (``mkg_slab_emit_normalized``), otherwise by a pass over the emitted values."""
    if normalize is not None and agg_mode != 0:
        raise ValueError("expand_forward: the normalisation belongs to the sum hop (agg_mode 0)")
    lib = N.load()
    dev = eng.dev
    E = eng.g.num_entities
    n = int(w_h.shape[-1])
    wf = w_h.detach().to(torch.float32).reshape(BL, n).contiguous()
    if check and keys.numel() and (int(keys.min()) < 0 or int(keys.max()) >= BL * E):
        raise RuntimeError("slab hop: a frontier key lies outside [B, L, E]")
    eng.ensure_store(BL)
    bounds = list(_windows(BL, eng.rows_per_window))
    out_k, out_v = [], []
    d = torch.zeros(BL, dtype=torch.float64, device=dev)
    st = N.stream_handle(dev)
    err = N.error_word(dev).data_ptr()
    nk = int(keys.numel())
    fused = normalize is not None and len(bounds) == 1 and nk > 0
    if nk == 0:
        ko, vo = torch.empty(0, dtype=torch.int64, device=dev), torch.empty(0, dtype=torch.float32, device=dev)
        if normalize is not None:
            return _normalized(ko, vo, d, [(0, 0)] * len(bounds), normalize, E, BL)
        return ko, vo, d, [(0, 0)] * len(bounds)
    k = keys.contiguous()
    v = vals.detach().to(torch.float32).contiguous()
    ws = N.workspace(lib.mkg_slab_expand_workspace_bytes(nk * eng.tile_groups[0][0]), dev)
    parts, pos = [], 0
    for r0, nr in bounds:  # every window takes the whole frontier and walks the entries of its rows
        rs = d[r0:r0 + nr].data_ptr() if agg_mode == 0 else None  # the expansions add their row sums
        win = eng.window(r0, nr)
        evs = []
        for gi, (nt, ptrs, recs) in enumerate(eng.tile_groups):  # one launch per group of tiles
            ev = _events(eng)  # (the same window; the first tile adds the identity messages)
            N.check(lib.mkg_slab_expand_tiles(nt, ctypes.addressof(ptrs), ctypes.addressof(recs), k.data_ptr(),
                                              v.data_ptr(), nk, wf.data_ptr(), n, int(gi == 0), int(agg_mode),
                                              ctypes.byref(win), eng.store.data_ptr(), rs, ws.data_ptr(), ws.numel(),
                                              err, st), "slab_expand")
            if ev is not None:
                ev[1].record()
                evs.append(ev)
        if fused:  # the whole of d is this window's: final once all-reduced
            _all_reduce(d, normalize[0])
            d32 = d.to(torch.float32)
            ko, vo, xo, dro = _collect(eng, win, (d32, normalize[1]))
        else:
            ko, vo = _collect(eng, win)
        out_k.append(ko)
        out_v.append(vo)
        parts.append((pos, pos + int(ko.numel())))
        pos += int(ko.numel())
        if evs:  # one hop of this window: frontier in + output out (12 B per key: 8 B key, 4 B
            # value), rule weights; its time is the sum over the tiles' expansions
            mine = _in_rows(k, E, r0, nr, len(bounds) == 1)
            eng.trace.append(("fwd", evs, graph_bytes(eng, mine) + 12 * int(mine.numel()) + 12 * int(ko.numel())
                              + nr * n * 4, len(eng.tiles)))
    ko, vo = (out_k[0], out_v[0]) if len(out_k) == 1 else (torch.cat(out_k), torch.cat(out_v))
    if fused:
        return ko, vo, d32, parts, xo, int(dro.item())
    if normalize is not None:
        return _normalized(ko, vo, d, parts, normalize, E, BL)
    return ko, vo, d, parts


def _normalized(keys, y, d, parts, normalize, E: int, BL: int):
    """expand_forward's normalised result by a separate pass: the row sums all-reduced, then
    ``mkg_mass_normalize``."""
    spec, threshold = normalize
    _all_reduce(d, spec)
    d32 = d.to(torch.float32)
    x, dropped = _mass_normalize(keys, y, E, BL, d32, threshold)
    return keys, y, d32, parts, x, dropped


def expand_backward(eng: SlabEngine, keys, vals, w_h, BL: int, keys_y, parts, put_grad, factor, grad_w64,
                    grad_edge):
    """Transposed walk of one hop: the frontier entries' fp64 gradient; adds to ``grad_w64``
    ([BL, n], fp64) and ``grad_edge`` ([T], fp32).  The hop's output ``keys_y`` came from the
    forward in the row-window parts ``parts``; ``put_grad(win, a, b)`` writes the output
    gradient of ``keys_y[a:b]`` into the store's window ``win`` before the window's walks (one
    per destination tile), which clears those keys after them."""
    lib = N.load()
    dev = eng.dev
    E = eng.g.num_entities
    n = int(w_h.shape[-1])
    wf = w_h.detach().to(torch.float32).reshape(BL, n).contiguous()
    bounds = list(_windows(BL, eng.rows_per_window))
    if len(parts) != len(bounds):
        raise RuntimeError("expand_backward: the store's windows changed since the forward")
    nk = int(keys.numel())
    gsp = torch.zeros(nk, dtype=torch.float64, device=dev)
    if nk == 0:
        return gsp
    st = N.stream_handle(dev)
    err = N.error_word(dev).data_ptr()
    ky = keys_y.contiguous()
    k = keys.contiguous()
    v = vals.detach().to(torch.float32).contiguous()
    ws = N.workspace(lib.mkg_slab_expand_workspace_bytes(nk * eng.tile_groups[0][0]), dev)
    for (r0, nr), (a, b) in zip(bounds, parts):  # every window takes the whole frontier
        win = eng.window(r0, nr)
        if b > a:
            put_grad(win, a, b)
        evs = []
        for gi, (nt, ptrs, recs) in enumerate(eng.tile_groups):  # one walk per group of tiles
            ev = _events(eng)  # (the first tile takes the identity messages)
            N.check(lib.mkg_slab_expand_backward_tiles(nt, ctypes.addressof(ptrs), ctypes.addressof(recs),
                                                       k.data_ptr(), v.data_ptr(), nk, wf.data_ptr(), n,
                                                       int(gi == 0), ctypes.byref(win), eng.store.data_ptr(),
                                                       ctypes.byref(factor), eng.g.num_facts, gsp.data_ptr(),
                                                       grad_w64.data_ptr(), N.ptr(grad_edge), ws.data_ptr(),
                                                       ws.numel(), err, st), "slab_expand_backward")
            if ev is not None:
                ev[1].record()
                evs.append(ev)
        if b > a:
            N.check(lib.mkg_slab_take(ctypes.byref(win), eng.store.data_ptr(), ky[a:b].data_ptr(), b - a, 1, None, 1,
                                      err, st), "slab_take")
        if evs:  # grad-in at the outputs, frontier re-read, grad-out, weights, edge grads (4 B per
            # edge-score gradient touched: at most one per message, at most T); time summed over tiles
            whole = len(bounds) == 1
            mine, mine_y = _in_rows(k, E, r0, nr, whole), _in_rows(ky, E, r0, nr, whole)
            local_deg = (eng.ptr[1:] - eng.ptr[:-1]).to(torch.int64)
            touched = min(eng.g.num_facts, int(local_deg[mine % E].sum())) if grad_edge is not None else 0
            eng.trace.append(("bwd", evs, graph_bytes(eng, mine) + 12 * int(mine_y.numel())
                              + 16 * int(mine.numel()) + nr * n * 4 + 4 * touched, len(eng.tiles)))
    return gsp


def sum_over_rules(eng: SlabEngine, keys, vals, B: int, L: int, take_max: bool = False,
                   entity_major_state: bool = False):
    """sum_sp_3d (fastlog_bridge.py:17-23): ``(b, l, e)`` entries (any order) added at ``(b, e)``
    (``take_max``: max_sp_3d's maximum instead); returns ascending ``b * E + e`` keys, their
    values and the inverse map (each entry's output position) for the backward.  One
    reduce-by-key (``mkg_reduce_by_key``: fp64 sums rounded once; maxima exact), or, for a state
    in entity-major order (``entity_major_state``: the output of a one-window store), the
    rule runs folded in place (``mkg_rule_sum``: fp32 sums in rule order) and one radix pass
    over the query."""
    E = eng.g.num_entities
    if entity_major_state:
        lib = N.load()
        dev = vals.device
        n = int(keys.numel())
        k = keys.contiguous()
        v = vals.detach().to(torch.float32).contiguous()
        ok = torch.empty(n, dtype=torch.int64, device=dev)
        ov = torch.empty(n, dtype=torch.float32, device=dev)
        pos = torch.empty(n, dtype=torch.int64, device=dev)
        cnt = torch.zeros(1, dtype=torch.int64, device=dev)
        ws = N.workspace(lib.mkg_rule_sum_workspace_bytes(n), dev)
        N.check(lib.mkg_rule_sum(N.ptr(k), N.ptr(v), n, E, L, B, 1 if take_max else 0, N.ptr(ok), N.ptr(ov),
                                 N.ptr(pos), cnt.data_ptr(), ws.data_ptr(), ws.numel(), N.error_word(dev).data_ptr(),
                                 N.stream_handle(dev)), "rule_sum")
        U = int(cnt.item())
        return ok[:U], ov[:U], pos
    from .sparse_reducers import _reduce
    keys2 = (keys // E) // L * E + keys % E
    uk, uv, inv, _ = _reduce(keys2, vals, 1 if take_max else 0, key_bits=max(1, int(B * E - 1).bit_length()))
    return uk, uv, inv


def spread_over_rules(g_out, inv):
    """Backward of ``sum_over_rules``: the gradient at every ``(b, l, e)`` entry is the output
    gradient at ``(b, e)``."""
    return g_out.to(torch.float32)[inv]


def _mass_normalize(keys, y, E: int, BL: int, d32, threshold: float):
    """(x = (y / d) * min(d, 1) per entry, number of entries the loop drops: zero or under the
    threshold)."""
    lib = N.load()
    dev = y.device
    x = torch.empty_like(y)
    dropped = torch.zeros(1, dtype=torch.int64, device=dev)
    N.check(lib.mkg_mass_normalize(keys.data_ptr(), y.data_ptr(), int(y.numel()), E, 0, BL, d32.data_ptr(),
                                   float(threshold), x.data_ptr(), dropped.data_ptr(), N.error_word(dev).data_ptr(),
                                   N.stream_handle(dev)), "mass_normalize")
    return x, int(dropped.item())


def _mass_normalize_grad_sums(keys, y, gx, E: int, BL: int, d32, spec):
    """Row sums of both terms of the mass normalisation's gradient, fp64 [2, BL], all-reduced
    over ranks."""
    lib = N.load()
    dev = y.device
    sums = torch.zeros((2, BL), dtype=torch.float64, device=dev)
    N.check(lib.mkg_mass_normalize_grad_sums(keys.data_ptr(), y.data_ptr(), gx.data_ptr(), int(y.numel()), E, 0, BL,
                                             d32.data_ptr(), sums.data_ptr(), N.error_word(dev).data_ptr(),
                                             N.stream_handle(dev)), "mass_normalize_grad_sums")
    return _all_reduce(sums, spec)


def _grad_putter(eng: SlabEngine, keys, y, gx, BL: int, d32, sums):
    """``put_grad(win, a, b)`` for ``expand_backward``: the normalisation's gradient of entries
    [a, b) written straight into the store's window (``mkg_mass_normalize_grad_put``)."""
    lib = N.load()
    dev = y.device
    E = eng.g.num_entities
    k, yy, g = keys.contiguous(), y.contiguous(), gx.contiguous()

    def put(win, a: int, b: int):
        N.check(lib.mkg_mass_normalize_grad_put(k[a:b].data_ptr(), yy[a:b].data_ptr(), g[a:b].data_ptr(), b - a, E, 0,
                                                BL, d32.data_ptr(), sums.data_ptr(), ctypes.byref(win),
                                                eng.store.data_ptr(), N.error_word(dev).data_ptr(),
                                                N.stream_handle(dev)), "mass_normalize_grad_put")
    return put


def _mass_normalize_grad(keys, y, gx, E: int, BL: int, d32, spec):
    """Gradient of the mass normalisation at its input: row sums of both terms in fp64
    (all-reduced over ranks), then the per-entry gradient."""
    lib = N.load()
    dev = y.device
    n = int(y.numel())
    st = N.stream_handle(dev)
    sums = _mass_normalize_grad_sums(keys, y, gx, E, BL, d32, spec)
    gy = torch.empty_like(y)
    N.check(lib.mkg_mass_normalize_grad(keys.data_ptr(), y.data_ptr(), gx.data_ptr(), n, E, 0, BL, d32.data_ptr(),
                                        sums.data_ptr(), gy.data_ptr(), st), "mass_normalize_grad")
    return gy


# ----------------------------------------------------------------------------- the loop
class _Hop:
    __slots__ = ("keys_in", "vals_in", "n_own", "offset", "prune_sel", "n_pre", "keys_y", "y", "d", "keep", "parts")


def _all_reduce(t, spec):
    if spec is not None and spec.world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, group=spec.group)
    return t


def _gather(keys, vals, spec):
    """The whole frontier on every rank: the ranks' lists concatenated in rank order (ranks own
    ascending entity ranges, so entity-major lists stay entity-major); returns (keys, values,
    this rank's offset in the concatenation, or None)."""
    if spec is None or spec.world == 1:
        return keys, vals, None
    import torch.distributed as dist
    from .sharded import _gather_counts
    counts = _gather_counts(int(keys.numel()), keys.device, spec.group)
    # keys and the values' fp32 bits in one [m, 2] int64 payload: one collective per hop
    m = max(max(counts), 1)
    pad = torch.zeros((m, 2), dtype=torch.int64, device=keys.device)
    pad[: keys.numel(), 0] = keys
    pad[: keys.numel(), 1] = vals.detach().to(torch.float32).contiguous().view(torch.int32).to(torch.int64)
    out = torch.empty((spec.world * m, 2), dtype=torch.int64, device=keys.device)
    dist.all_gather_into_tensor(out, pad, group=spec.group)
    rows = torch.cat([out[r * m: r * m + c] for r, c in enumerate(counts)])
    k_all = rows[:, 0].contiguous()
    v_all = rows[:, 1].to(torch.int32).view(torch.float32)
    return k_all, v_all, sum(counts[: spec.rank])


def _prune(keys, vals, E, topk_nodes):
    """prune_sparse3d_active_entities (drum.py:54-80) on the whole frontier (every rank holds
    it after the gather, so every rank selects the same entries)."""
    if topk_nodes <= 0:
        return keys, vals, None
    from .sparse_loop import _prune as prune_state
    return prune_state(keys, vals, E, topk_nodes)


class SlabHopLoop(autograd.Function):
    """``(w_hops [K, B, L, n], edge_scores [T]) -> (keys b * E + e, values, messages [K])`` of the
    uncapped sum hop loop on the key-slab engine; gradients for ``w_hops`` and ``edge_scores``.
    With a ``ShardSpec`` each rank returns its own entities' part of the result, and every rank
    receives the full gradients."""

    @staticmethod
    def forward(ctx, w_hops, edge_scores, heads, eng: SlabEngine, mask, is_score: bool, scale: float,
                topk_nodes: int, threshold: float, spec):
        N.require_cuda(w_hops, "w_hops")
        K, B, L, n = (int(s) for s in w_hops.shape)
        g = eng.g
        E = g.num_entities
        if n != 2 * g.num_relations + 1:
            raise ValueError(f"w_hops has {n} channels, expected 2R+1 = {2 * g.num_relations + 1}")
        dev = eng.dev
        BL = B * L
        eng.set_edge_factor(mask, edge_scores.detach() if edge_scores is not None else None, is_score, scale)
        factor_write = g.factor_writes
        wf = w_hops.detach().to(torch.float32).contiguous()
        hd = heads.to(device=dev, dtype=torch.int64)
        if bool(((hd < 0) | (hd >= E)).any()):
            raise ValueError(f"query heads must lie in [0, {E})")
        src = hd.repeat_interleave(L)
        keys = torch.arange(BL, device=dev) * E + src
        if eng.lo > 0 or eng.hi < E:  # a destination range: this rank's heads only
            keys = keys[(src >= eng.lo) & (src < eng.hi)]
        keys, _ = entity_major(keys, keys, E, BL)
        vals = torch.ones(keys.numel(), dtype=torch.float32, device=dev)
        hops, msgs = [], []
        for h in range(K):
            st = _Hop()
            st.n_own = int(keys.numel())
            k_all, v_all, st.offset = _gather(keys, vals, spec)
            st.n_pre = int(k_all.numel())
            k_all, v_all, st.prune_sel = _prune(k_all, v_all, E, int(topk_nodes))
            st.keys_in, st.vals_in = k_all, v_all
            msgs.append(eng.full_degree[k_all % E].sum())
            ky, y, d32, st.parts, x, dropped = expand_forward(eng, k_all, v_all, wf[h], BL, check=False,
                                                               normalize=(spec, threshold))
            st.keys_y, st.y, st.d, st.keep = ky, y, d32, None
            if dropped:  # some results are zero or under the threshold: the loop drops them
                keep = x != 0
                if threshold > 0:
                    keep &= x >= threshold
                st.keep = keep
                keys, vals = ky[keep], x[keep]
            else:
                keys, vals = ky, x
            hops.append(st)
        out_keys, out_vals, inv = sum_over_rules(eng, keys, vals, B, L,
                                                 entity_major_state=eng.rows_per_window >= BL)
        N.raise_device_errors(dev)  # an out-of-range index any kernel of the forward met
        ctx.hops, ctx.eng, ctx.spec = hops, eng, spec
        ctx.factor_write = factor_write
        ctx.rule_inv = inv
        ctx.wf, ctx.shape = wf, (K, B, L, n)
        ctx.mask, ctx.is_score, ctx.scale = mask, bool(is_score), float(scale)
        ctx.edge_scores = edge_scores.detach() if edge_scores is not None else None
        ctx.want_edge = edge_scores is not None and ctx.needs_input_grad[1]
        ctx.edge_shape = tuple(edge_scores.shape) if edge_scores is not None else None
        ctx.edge_dtype = edge_scores.dtype if edge_scores is not None else None
        ctx.mark_non_differentiable(out_keys)
        m_t = torch.stack(msgs) if msgs else torch.zeros(0, dtype=torch.int64, device=dev)
        ctx.mark_non_differentiable(m_t)
        return out_keys, out_vals, m_t

    @staticmethod
    def backward(ctx, _g_keys, g_vals, _g_msgs):
        eng, spec = ctx.eng, ctx.spec
        g = eng.g
        E = g.num_entities
        K, B, L, n = ctx.shape
        BL = B * L
        dev = eng.dev
        # the factor field may have been rewritten since the forward (another loop on this graph)
        if g.factor_writes != ctx.factor_write:
            eng.set_edge_factor(ctx.mask, ctx.edge_scores, ctx.is_score, ctx.scale)
        keep_alive = []
        factor = N.edge_factor(ctx.mask, ctx.edge_scores, ctx.is_score, ctx.scale, keep_alive)
        grad_w64 = torch.zeros((K, BL, n), dtype=torch.float64, device=dev)
        grad_edge = torch.zeros(g.num_facts, dtype=torch.float32, device=dev) if ctx.want_edge else None
        g_state = spread_over_rules(g_vals, ctx.rule_inv)
        for h in range(K - 1, -1, -1):
            st = ctx.hops[h]
            if st.keep is None:
                gx = g_state.to(torch.float32).contiguous()
            else:
                gx = torch.zeros_like(st.y)
                gx[st.keep] = g_state
            sums = _mass_normalize_grad_sums(st.keys_y, st.y, gx, E, BL, st.d, spec)
            put = _grad_putter(eng, st.keys_y, st.y, gx, BL, st.d, sums)
            gsp = expand_backward(eng, st.keys_in, st.vals_in, ctx.wf[h], BL, st.keys_y, st.parts, put, factor,
                                  grad_w64[h], grad_edge)
            if st.prune_sel is not None:  # back to the frontier before the prune
                full = torch.zeros(st.n_pre, dtype=gsp.dtype, device=dev)
                full[st.prune_sel] = gsp
                gsp = full
            if st.offset is not None:  # several ranks: sum the partials, keep this rank's entries
                _all_reduce(gsp, spec)
                gsp = gsp[st.offset: st.offset + st.n_own]
            g_state = gsp.to(torch.float32)
        _all_reduce(grad_w64, spec)
        if grad_edge is not None:
            _all_reduce(grad_edge, spec)
        N.raise_device_errors(dev)
        gw = grad_w64.to(torch.float32).view(K, B, L, n)
        ge = grad_edge.view(ctx.edge_shape).to(ctx.edge_dtype) if grad_edge is not None else None
        return gw, ge, None, None, None, None, None, None, None, None


def slab_engine(graph: DeviceGraph) -> SlabEngine:
    """The whole-range engine of ``graph``, made once and kept with it."""
    eng = getattr(graph, "_slab_engine", None)
    if eng is None:
        eng = SlabEngine(graph)
        graph._slab_engine = eng
    return eng


def slab_proof_scores(engine: SlabEngine, heads: torch.Tensor, w_hops: torch.Tensor,
                      edge_scores: torch.Tensor | None, mask: torch.Tensor | None = None, is_score: bool = True,
                      scale: float = 1.0, topk_nodes: int = 0, threshold: float = 0.0, spec=None,
                      dense: bool = False):
    """The loop's result as a sparse ``[B, E]`` tensor (``dense=True``: dense; with ``spec``:
    this rank's entities) and the per-hop message counts."""
    K, B, L, n = (int(s) for s in w_hops.shape)
    E = engine.g.num_entities
    keys, vals, msgs = SlabHopLoop.apply(w_hops, edge_scores, heads, engine, mask, is_score, scale, int(topk_nodes),
                                         float(threshold), spec)
    out = torch.sparse_coo_tensor(torch.stack([keys // E, keys % E]), vals, (B, E), is_coalesced=True)
    return (out.to_dense() if dense else out), msgs


@torch.no_grad()
def slab_decode_max(engine: SlabEngine, heads: torch.Tensor, w_hops: torch.Tensor, topk: int,
                    edge_scores: torch.Tensor | None, mask: torch.Tensor | None = None, is_score: bool = True,
                    scale: float = 1.0, msgs_out: list | None = None):
    """The max-aggregation loop of src/model_mmDRUM_kernel_sp.py:388-445, uncapped, on the
    key-slab store: per hop every key keeps its largest message (the op with ``agg_mode=1``
    followed by ``sparse3d_max(ind, ori, inv)``: the value of a maximum does not depend on which
    tied message wins), then ``norm_sp_3d`` (row sums added one by one in key order, as the
    reference's CPU ``index_put_``, clamped at 1e-7; zeros dropped); after the last hop the max
    over rules (``norm_sp_3d_max``); then the decode order of ordered_tail_scores
    (decode_core.py:350-363) on the bounded scores, ``topk`` per query.  Bit-exact with the
    reference.  Returns (keys ``b * E + e`` ascending, raw scores, tails [B, topk] -1 padded,
    bounded scores [B, topk], counts [B]); with ``msgs_out`` the message count of every hop is
    appended (device scalars)."""
    from .proof import sparse_topk
    N.require_cuda(w_hops, "w_hops")
    K, B, L, n = (int(s) for s in w_hops.shape)
    eng = engine
    E = eng.g.num_entities
    if eng.lo != 0 or eng.hi != E:
        raise ValueError("slab_decode_max runs on a whole-range engine")
    dev = eng.dev
    BL = B * L
    eng.set_edge_factor(mask, edge_scores.detach() if edge_scores is not None else None, is_score, scale)
    wf = w_hops.detach().to(torch.float32).contiguous()
    hd = heads.to(device=dev, dtype=torch.int64)
    if bool(((hd < 0) | (hd >= E)).any()):
        raise ValueError(f"query heads must lie in [0, {E})")
    keys = torch.arange(BL, device=dev) * E + hd.repeat_interleave(L)
    keys, _ = entity_major(keys, keys, E, BL)
    vals = torch.ones(BL, dtype=torch.float32, device=dev)
    for h in range(K):
        if msgs_out is not None:
            msgs_out.append(eng.full_degree[keys % E].sum())
        ky, y, _, _ = expand_forward(eng, keys, vals, wf[h], BL, check=False, agg_mode=1)
        rows = ky // E
        # each row's entries in ascending entity order (a stable sort by row of the
        # entity-major list), summed one by one in that order
        # (rows fit 16 bits for up to 32,767 (b, l) rows: a two-pass radix sort)
        by_row = torch.sort(rows.to(torch.int16) if BL <= 32767 else rows, stable=True)
        seg = torch.searchsorted(by_row.values.to(torch.int64), torch.arange(BL + 1, device=dev, dtype=torch.int64))
        d = N.segment_sum(seg, y[by_row.indices], ordered=True).clamp(min=1e-7)
        x = y / d[rows]
        keep = torch.nonzero(x != 0, as_tuple=True)[0]
        keys, vals = ky[keep], x[keep]
    out_keys, out_vals, _ = sum_over_rules(eng, keys, vals, B, L, take_max=True,
                                           entity_major_state=eng.rows_per_window >= BL)
    N.raise_device_errors(dev)
    tails, scores, counts = sparse_topk(out_keys, out_vals, B, E, int(topk))
    return out_keys, out_vals, tails, scores, counts
