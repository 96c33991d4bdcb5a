"""The bridge reducers on the device: the reference's helper names, arguments and results
(sum_sp_3d / sum_sparse3d_concat, src/fastlog_bridge.py:17-42; max_sp_3d / sparse3d_max /
norm_sp_3d / norm_sp_3d_max, src/model_mmDRUM_kernel_sp.py:39-270; normalize_sparse3d /
prune_sparse3d_active_entities, drum.py:31-80; bound_sparse_scores, proof.py:642-649) for a
caller that drives single hops of ``FastLogFunctionSparse3DTopK`` itself.

Every reduction over keys is one ``mkg_reduce_by_key`` call (stable radix sort of the flat
keys, fp64 run sums or first-wins run maxima, csrc/mkg_reduce.cu); the per-(b, l) sums of the
normalisations are ``mkg_segment_sum_ordered`` (fp32, added in key order, the order of the
reference's CPU ``index_put_``).  Inputs and results are torch sparse COO tensors on a CUDA
device; gradients flow through the values (a sum spreads its gradient back over its inputs,
a maximum hands it to its winning entry, a row sum to every entry of the row).

Ties: ``max_sp_3d`` keeps the lowest rule ``l``; ``sparse3d_max`` the earliest argument;
``prune_sparse3d_active_entities`` ranks equal entity scores by entity id (``torch.topk``'s
tie order is unspecified in the reference).
"""
from __future__ import annotations

import torch
from torch import autograd

from . import _native as N


# ----------------------------------------------------------------------------- flat keys
def _flat(s: torch.Tensor):
    """(flat keys, values, shape) of a sparse COO tensor: keys in row-major order of its dims."""
    N.require_cuda(s, "a sparse state")
    s = s.coalesce()
    idx = s.indices()
    shape = tuple(int(x) for x in s.shape)
    key = idx[0].clone()
    for d in range(1, len(shape)):
        key = key * shape[d] + idx[d]
    return key, s.values(), shape


def _unflat(keys: torch.Tensor, shape) -> torch.Tensor:
    rows = []
    rest = keys
    for d in range(len(shape) - 1, 0, -1):
        rows.append(rest % shape[d])
        rest = rest // shape[d]
    rows.append(rest)
    return torch.stack(rows[::-1]) if keys.numel() else torch.empty((len(shape), 0), dtype=torch.int64,
                                                                      device=keys.device)


def _coo(keys, vals, shape) -> torch.Tensor:
    return torch.sparse_coo_tensor(_unflat(keys, shape), vals, shape, is_coalesced=True)


def _reduce(keys: torch.Tensor, vals: torch.Tensor, mode: int, key_bits: int | None = None):
    """(unique keys ascending, reduced values, inverse [n], arg [U]) of ``mkg_reduce_by_key``;
    ``key_bits`` bounds the keys (default: read from the largest key)."""
    lib = N.load()
    dev = vals.device
    n = int(keys.numel())
    k = keys.to(torch.int64).contiguous()
    v = vals.detach().to(torch.float32).contiguous()
    ok = torch.empty(n, dtype=torch.int64, device=dev)
    ov = torch.empty(n, dtype=torch.float32, device=dev)
    inv = torch.empty(n, dtype=torch.int64, device=dev)
    arg = torch.empty(n, dtype=torch.int64, device=dev) if mode == 1 else None
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    bits = key_bits if key_bits is not None else (max(1, int(k.max()).bit_length()) if n else 1)
    ws = N.workspace(lib.mkg_reduce_by_key_workspace_bytes(n), dev)
    N.check(lib.mkg_reduce_by_key(k.data_ptr(), v.data_ptr(), n, mode, min(bits, 63), ok.data_ptr(), ov.data_ptr(),
                                  cnt.data_ptr(), inv.data_ptr(), N.ptr(arg), ws.data_ptr(), ws.numel(),
                                  N.error_word(dev).data_ptr(), N.stream_handle(dev)), "reduce_by_key")
    U = int(cnt.item())
    N.raise_device_errors(dev)
    return ok[:U], ov[:U], inv, (arg[:U] if arg is not None else None)


class _SumByKey(autograd.Function):
    @staticmethod
    def forward(ctx, keys, vals):
        uk, uv, inv, _ = _reduce(keys, vals, 0)
        ctx.save_for_backward(inv)
        ctx.mark_non_differentiable(uk)
        return uk, uv.to(vals.dtype)

    @staticmethod
    def backward(ctx, _gk, g):
        inv, = ctx.saved_tensors
        return None, g[inv]


class _MaxByKey(autograd.Function):
    @staticmethod
    def forward(ctx, keys, vals):
        uk, uv, _, arg = _reduce(keys, vals, 1)
        ctx.save_for_backward(arg)
        ctx.n = int(vals.numel())
        ctx.mark_non_differentiable(uk)
        return uk, uv.to(vals.dtype)

    @staticmethod
    def backward(ctx, _gk, g):
        arg, = ctx.saved_tensors
        out = torch.zeros(ctx.n, dtype=g.dtype, device=g.device)
        out[arg] = g
        return None, out


class _RowSum(autograd.Function):
    """Per-row sums of ``vals`` over rows ``[seg[r], seg[r + 1])``, added in index order (fp32)."""

    @staticmethod
    def forward(ctx, vals, seg, rows):
        ctx.save_for_backward(rows)
        return N.segment_sum(seg, vals, ordered=True).to(vals.dtype)

    @staticmethod
    def backward(ctx, g):
        rows, = ctx.saved_tensors
        return g[rows], None, None


def _rows_of(keys: torch.Tensor, E: int, nrows: int):
    """Row of every 3-D key ``(b * L + l) * E + e`` and the row boundaries of the sorted keys."""
    rows = keys // E
    seg = torch.searchsorted(rows, torch.arange(nrows + 1, device=keys.device, dtype=rows.dtype))
    return rows, seg


def _empty_like_state(shape, dev, dtype=torch.float32):
    return _coo(torch.empty(0, dtype=torch.int64, device=dev), torch.empty(0, dtype=dtype, device=dev), shape)


# ----------------------------------------------------------------------------- sums
def sum_sparse3d_concat(*states: torch.Tensor) -> torch.Tensor:
    """Union-sum of sparse [B, L, E] states (a state alone is returned as it is)."""
    live = [s for s in states if s._nnz() > 0]
    if not live:
        return _empty_like_state(tuple(states[0].shape), states[0].device, states[0].dtype)
    if len(live) == 1:
        return live[0]
    parts = [_flat(s) for s in live]
    shape = parts[0][2]
    keys, vals = _SumByKey.apply(torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts]))
    return _coo(keys, vals, shape)


def sum_sp_3d(s: torch.Tensor) -> torch.Tensor:
    """Sum over rules: [B, L, E] -> [B, E]."""
    key, val, (B, L, E) = _flat(s)
    key2 = (key // (L * E)) * E + key % E
    keys, vals = _SumByKey.apply(key2, val)
    return _coo(keys, vals, (B, E))


# ----------------------------------------------------------------------------- maxima
def _drop_zeros(keys, vals):
    keep = torch.nonzero(vals.detach() != 0, as_tuple=True)[0]
    return keys[keep], vals[keep]


def max_sp_3d(s: torch.Tensor) -> torch.Tensor:
    """Max over rules: [B, L, E] -> [B, E]; equal maxima keep the lowest rule; zeros dropped."""
    key, val, (B, L, E) = _flat(s)
    if key.numel() == 0:
        return _empty_like_state((B, E), val.device, val.dtype)
    # entries come in (b, l, e) order, so equal (b, e) keys meet in ascending l: first wins
    keys, vals = _MaxByKey.apply((key // (L * E)) * E + key % E, val)
    return _coo(*_drop_zeros(keys, vals), (B, E))


def sparse3d_max(*states: torch.Tensor) -> torch.Tensor:
    """Element-wise max of [B, L, E] states; equal maxima keep the earliest argument; zeros
    dropped."""
    parts = [_flat(s) for s in states]
    shape = parts[0][2]
    keys = torch.cat([p[0] for p in parts])
    if keys.numel() == 0:
        return _empty_like_state(shape, states[0].device, states[0].dtype)
    k, v = _MaxByKey.apply(keys, torch.cat([p[1] for p in parts]))
    return _coo(*_drop_zeros(k, v), shape)


# ----------------------------------------------------------------------------- normalisations
def norm_sp_3d(s: torch.Tensor, detach_norm: bool = False) -> torch.Tensor:
    """values / clamp(per-(b, l) sum, 1e-7), zeros dropped."""
    key, val, (B, L, E) = _flat(s)
    if key.numel() == 0:
        return _empty_like_state((B, L, E), val.device, val.dtype)
    rows, seg = _rows_of(key, E, B * L)
    denom = _RowSum.apply(val, seg, rows).clamp(min=1e-7)
    if detach_norm:
        denom = denom.detach()
    out = val / denom[rows]
    return _coo(*_drop_zeros(key, out), (B, L, E))


def norm_sp_3d_max(s: torch.Tensor, dropout=None, detach_norm: bool = False) -> torch.Tensor:
    """norm_sp_3d, the optional dropout on the values, then max_sp_3d."""
    s = norm_sp_3d(s, detach_norm=detach_norm)
    if dropout is not None and float(getattr(dropout, "p", 0.0) or 0.0) > 0.0:
        key, val, shape = _flat(s)
        s = _coo(key, dropout(val), shape)
    return max_sp_3d(s)


def normalize_sparse3d(state: torch.Tensor, eps: float, availability: str) -> torch.Tensor:
    """Per-(b, l) normalisation: zeros dropped, ``d`` = the row's sum (at least ``eps`` when
    eps > 0), values / d, times min(d, 1) for the "mass" availability; zeros dropped."""
    if availability not in ("mass", "none"):
        raise ValueError(f"unknown proof_norm_availability: {availability}")
    key, val, (B, L, E) = _flat(state)
    key, val = _drop_zeros(key, val)
    if key.numel() == 0:
        return _empty_like_state((B, L, E), state.device, state.dtype)
    rows, seg = _rows_of(key, E, B * L)
    d = _RowSum.apply(val, seg, rows)
    if eps > 0:
        d = d.clamp_min(eps)
    out = val / d[rows]
    if availability == "mass":
        out = out * d.clamp_max(1.0)[rows]
    return _coo(*_drop_zeros(key, out), (B, L, E))


# ----------------------------------------------------------------------------- prune, bound
def prune_sparse3d_active_entities(state: torch.Tensor, topk_nodes: int) -> torch.Tensor:
    """Keeps the entries of the ``topk_nodes`` entities with the largest summed |value| over the
    whole state (equal sums: lower entity id), unless the state has at most ``topk_nodes``
    entries."""
    if topk_nodes <= 0 or state._nnz() <= topk_nodes:
        return state
    key, val, (B, L, E) = _flat(state)
    ent = key % E
    score = torch.zeros(E, dtype=val.dtype, device=val.device).index_add_(0, ent, val.detach().abs())
    k = min(int(topk_nodes), E)
    chosen = torch.sort(score, descending=True, stable=True).indices[:k]
    keep_ent = torch.zeros(E, dtype=torch.bool, device=val.device)
    keep_ent[chosen] = True
    sel = torch.nonzero(keep_ent[ent], as_tuple=True)[0]
    if sel.numel() == key.numel():
        return state
    return _coo(key[sel], val[sel], (B, L, E))


def bound_sparse_scores(raw: torch.Tensor) -> torch.Tensor:
    """1 - exp(-max(x, 0)) on the values (dense input: elementwise); exp rounded from double,
    as the device decode computes it."""
    def bound(x):
        return 1.0 - torch.exp(-x.clamp_min(0.0).double()).to(x.dtype)
    if not raw.is_sparse:
        return bound(raw)
    key, val, shape = _flat(raw)
    return _coo(key, bound(val), shape)
