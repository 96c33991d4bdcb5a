"""Decode candidates on the device, with the reference's decode entry points.

The reference decodes a relation batch by batch (decode_core.py:394-420,
``iter_decode_candidate_batches``): per proof microbatch ``kernel_sparse_scores`` (sum
mode), ``bound_sparse_scores`` (proof.py:642-649), ``sparse_candidate_rows`` (proof.py:729-758:
the sparse scores copied to the host and split per row) and, per row, ``ordered_tail_scores``
(decode_core.py:350-363: ``np.lexsort((tails, -scores))``, score descending then tail
ascending).  Here the bound and the ordering run on the device (``proof.sparse_topk``, or the
top-k kernel ``mkg_decode_topk`` for dense scores and caps up to 1024) and one copy brings the
ordered rows to the host, so ``ordered_tail_scores`` applied by a caller leaves them as they are.
The bound's exponential is rounded from double (one ulp from torch's float32 exp at most).
"""
from __future__ import annotations

import numpy as np
import torch

from .proof import decode_topk, kernel_sparse_scores, sparse_topk

_TOPK_KERNEL_MAX = 1024  # kTopkMax of mkg_decode_topk


def ordered_candidates(raw: torch.Tensor, cap: int = 0):
    """Candidates of raw scores ``[B, E]`` (dense, or sparse COO; non-zero entries) in decode
    order with bounded scores: (tails [B, k] int64 -1 padded, scores [B, k] f32, counts [B]);
    ``k = cap`` when ``cap > 0``, else the longest row (every candidate)."""
    B, E = (int(s) for s in raw.shape)
    if not raw.is_sparse and 0 < cap <= _TOPK_KERNEL_MAX:
        return decode_topk(raw, int(cap))
    if raw.is_sparse:
        r = raw.coalesce()
        idx, vals = r.indices(), r.values()
        keep = vals != 0
        keys = (idx[0] * E + idx[1])[keep]
        vals = vals[keep]
    else:
        nz = raw.nonzero(as_tuple=False)
        keys = nz[:, 0] * E + nz[:, 1]
        vals = raw[nz[:, 0], nz[:, 1]]
    k = int(cap)
    if k <= 0:
        k = int(torch.bincount(keys // E, minlength=B).max().item()) if keys.numel() else 0
    if k == 0:
        dev = raw.device
        return (torch.full((B, 0), -1, dtype=torch.int64, device=dev), torch.zeros((B, 0), device=dev),
                torch.zeros(B, dtype=torch.int64, device=dev))
    return sparse_topk(keys, vals.float(), B, E, k)


def candidate_rows(tails: torch.Tensor, scores: torch.Tensor, counts: torch.Tensor) -> dict:
    """{row: (tails int64, scores float32)} for the rows with candidates (one device-to-host copy),
    the shape ``sparse_candidate_rows`` returns."""
    t, s, c = tails.cpu().numpy(), scores.cpu().numpy().astype(np.float32), counts.cpu().numpy()
    return {int(r): (t[r, : c[r]].astype(np.int64), s[r, : c[r]]) for r in np.nonzero(c)[0]}


def sparse_candidate_rows(scores: torch.Tensor) -> dict:
    """proof.py:729-758: {row: (tails, values)} of a sparse ``[B, E]`` score tensor, rows in
    ascending order, each row's entries in ascending tail order as the coalesced tensor holds
    them (values unchanged)."""
    s = scores.coalesce()
    idx, val = s.indices(), s.values()
    if idx.numel() == 0:
        return {}
    rows, tails = idx[0].cpu().numpy().astype(np.int64), idx[1].cpu().numpy().astype(np.int64)
    vals = val.detach().to(torch.float32).cpu().numpy()
    bounds = np.flatnonzero(np.diff(rows)) + 1
    out = {}
    for a, b in zip(np.concatenate([[0], bounds]), np.concatenate([bounds, [rows.size]])):
        out[int(rows[a])] = (tails[a:b], vals[a:b])
    return out


def iter_decode_candidate_batches(model, heads: torch.Tensor, relations: torch.Tensor, graph, args):
    """decode_core.py:394-420: per proof microbatch (``args.decode_proof_microbatch_size``, 0 =
    one batch) yields ``(row_start, row_end, rows)``, ``rows`` = {row within the microbatch:
    (tails, bounded scores)} with every candidate, already in decode order."""
    total = int(heads.shape[0])
    micro = int(getattr(args, "decode_proof_microbatch_size", 0) or 0)
    if micro <= 0:
        micro = max(total, 1)
    with torch.no_grad():
        for a in range(0, total, micro):
            b = min(a + micro, total)
            raw = kernel_sparse_scores(model, heads[a:b], relations[a:b], graph, args, is_training=False, dense=True)
            tails, scores, counts = ordered_candidates(raw, 0)
            yield a, b, candidate_rows(tails, scores, counts)
