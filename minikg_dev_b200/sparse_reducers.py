"""Reducers of the bridge / proof loop on torch sparse COO tensors.

Same names, arguments and results as the reference helpers; they are what a caller that
keeps the reference's per-hop loop composes around ``FastLogFunctionSparse3DTopK``:

* ``sum_sp_3d``, ``sum_sparse3d_concat`` — src/fastlog_bridge.py:17-42;
* ``max_sp_3d`` (ties → lowest rule), ``sparse3d_max`` (ties → earliest argument),
  ``norm_sp_3d``, ``norm_sp_3d_max`` — src/model_mmDRUM_kernel_sp.py:39-270;
* ``normalize_sparse3d``, ``prune_sparse3d_active_entities`` — drum.py:31-80
  (the prune breaks equal entity scores towards the lower entity id);
* ``bound_sparse_scores`` — proof.py:642-649.

The fused hop loop (``minikg_dev_b200.proof``) performs the same reductions inside its CUDA
kernels; these torch versions exist for callers that drive single hops.
"""
from __future__ import annotations

import torch


def _unique_coo(idx, val, shape):
    return torch.sparse_coo_tensor(idx, val, shape, is_coalesced=True)


def sum_sp_3d(s: torch.Tensor) -> torch.Tensor:
    s = s.coalesce()
    idx = s.indices()
    B, _, E = s.shape
    return torch.sparse_coo_tensor(torch.stack([idx[0], idx[2]]), s.values(), [B, E]).coalesce()


def sum_sparse3d_concat(*states: torch.Tensor) -> torch.Tensor:
    states = [s.coalesce() for s in states]
    non_empty = [s for s in states if s._nnz() > 0]
    if not non_empty:
        dev = states[0].device
        e = torch.empty(0, dtype=torch.long, device=dev)
        return _unique_coo(torch.stack([e, e, e]), torch.empty(0, dtype=states[0].values().dtype, device=dev),
                           states[0].shape)
    if len(non_empty) == 1:
        return non_empty[0]
    idx = torch.cat([s.indices() for s in non_empty], dim=1)
    val = torch.cat([s.values() for s in non_empty])
    return torch.sparse_coo_tensor(idx, val, non_empty[0].shape).coalesce()


def _max_over_slots(key, slot, val, slot_count):
    """Max of ``val`` per ``key``; among equal maxima the smallest ``slot`` wins."""
    order = torch.argsort(key * slot_count + slot)
    sk = (key * slot_count + slot)[order] // slot_count
    sv = val.detach()[order]
    uniq, inv = torch.unique_consecutive(sk, return_inverse=True)
    mx = torch.full((uniq.shape[0],), float("-inf"), device=val.device, dtype=val.dtype)
    mx.scatter_reduce_(0, inv, sv, reduce="amax", include_self=True)
    pos = torch.arange(sv.shape[0], device=val.device)
    cand = torch.where(sv == mx[inv], pos, torch.full_like(pos, sv.shape[0]))
    arg = torch.full((uniq.shape[0],), sv.shape[0], device=val.device, dtype=torch.long)
    arg.scatter_reduce_(0, inv, cand, reduce="amin", include_self=True)
    return uniq, order[arg]


def max_sp_3d(s: torch.Tensor) -> torch.Tensor:
    s = s.coalesce()
    idx, val = s.indices(), s.values()
    B, L, E = s.shape
    if val.numel() == 0:
        e = torch.empty(0, dtype=torch.long, device=val.device)
        return _unique_coo(torch.stack([e, e]), val, [B, E])
    uniq, raw = _max_over_slots(idx[0] * E + idx[2], idx[1], val, L)
    out = val[raw]
    keep = out != 0
    uniq, out = uniq[keep], out[keep]
    return _unique_coo(torch.stack([uniq // E, uniq % E]), out, [B, E])


def sparse3d_max(*states: torch.Tensor) -> torch.Tensor:
    states = [s.coalesce() for s in states]
    B, L, E = states[0].shape
    keys, vals, slots = [], [], []
    for i, s in enumerate(states):
        idx = s.indices()
        keys.append(idx[0] * (L * E) + idx[1] * E + idx[2])
        vals.append(s.values())
        slots.append(torch.full_like(keys[-1], i))
    key, val, slot = torch.cat(keys), torch.cat(vals), torch.cat(slots)
    if val.numel() == 0:
        e = torch.empty(0, dtype=torch.long, device=val.device)
        return _unique_coo(torch.stack([e, e, e]), val, [B, L, E])
    uniq, raw = _max_over_slots(key, slot, val, len(states))
    out = val[raw]
    keep = out != 0
    uniq, out = uniq[keep], out[keep]
    return _unique_coo(torch.stack([uniq // (L * E), (uniq % (L * E)) // E, uniq % E]), out, [B, L, E])


def norm_sp_3d(s: torch.Tensor, detach_norm: bool = False) -> torch.Tensor:
    s = s.coalesce()
    idx, val = s.indices(), s.values()
    B, L, _ = s.shape
    denom = torch.zeros(B, L, device=val.device, dtype=val.dtype)
    denom.index_put_((idx[0], idx[1]), val, accumulate=True)
    denom = denom.clamp(min=1e-7)
    dn = denom.detach() if detach_norm else denom
    out = val / dn[idx[0], idx[1]]
    keep = out != 0
    return _unique_coo(idx[:, keep], out[keep], s.shape)


def norm_sp_3d_max(s: torch.Tensor, dropout=None, detach_norm: bool = False) -> torch.Tensor:
    s = norm_sp_3d(s, detach_norm=detach_norm)
    if dropout is not None and float(getattr(dropout, "p", 0.0) or 0.0) > 0.0:
        s = _unique_coo(s.indices(), dropout(s.values()), s.shape)
    return max_sp_3d(s)


def normalize_sparse3d(state: torch.Tensor, eps: float, availability: str) -> torch.Tensor:
    state = state.coalesce()
    idx, val = state.indices(), state.values()
    keep = val != 0
    idx, val = idx[:, keep], val[keep]
    B, L, _ = state.shape
    denom = torch.zeros(B, L, device=val.device, dtype=val.dtype)
    denom.index_put_((idx[0], idx[1]), val, accumulate=True)
    if eps > 0:
        denom = denom.clamp_min(eps)
    out = val / denom[idx[0], idx[1]]
    if availability == "mass":
        out = out * denom.clamp_max(1.0)[idx[0], idx[1]]
    elif availability != "none":
        raise ValueError(f"unknown proof_norm_availability: {availability}")
    keep = out != 0
    return torch.sparse_coo_tensor(idx[:, keep], out[keep], state.shape, device=val.device).coalesce()


def prune_sparse3d_active_entities(state: torch.Tensor, topk_nodes: int) -> torch.Tensor:
    if topk_nodes <= 0:
        return state
    state = state.coalesce()
    idx, val = state.indices(), state.values()
    if val.numel() <= topk_nodes:
        return state
    E = state.shape[2]
    k = min(int(topk_nodes), int(E))
    score = torch.zeros(E, dtype=val.dtype, device=val.device)
    score.index_add_(0, idx[2], val.detach().abs())
    # stable descending sort: equal scores keep ascending entity order
    order = torch.sort(score, descending=True, stable=True).indices
    keep_entity = torch.zeros(E, dtype=torch.bool, device=val.device)
    keep_entity[order[:k]] = True
    keep = keep_entity[idx[2]]
    if bool(keep.all().item()):
        return state
    return torch.sparse_coo_tensor(idx[:, keep], val[keep], state.shape, device=val.device).coalesce()


def bound_sparse_scores(raw: torch.Tensor) -> torch.Tensor:
    if not raw.is_sparse:
        return 1.0 - torch.exp(-raw.clamp_min(0.0))
    raw = raw.coalesce()
    values = 1.0 - torch.exp(-raw.values().clamp_min(0.0))
    return torch.sparse_coo_tensor(raw.indices(), values, raw.shape, device=values.device).coalesce()
