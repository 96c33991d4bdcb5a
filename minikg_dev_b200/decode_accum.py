"""The decode accumulator on the device: the best-k cut of every ordered candidate row.

``_OracleRelationAccumulator.add_row`` (decode.py:72-116) takes one query row at a time on
the host: the candidate tails in decode order (score descending, tail ascending), the query's
true tails and its base (already supplied) tails; it picks the cut k that maximises
(base true + new true) - new wrong (ties: more true, then fewer wrong, then the smaller k,
``_oracle_best_k``, decode.py:45-69) and accumulates candidate / selection / new-fact counters.

``DecodeAccumulator.add_rows`` does the same for a whole batch of rows at once, on the
tensors the device decode produces (``tails [B, k]`` padded with -1 and ``counts [B]``, e.g.
from ``proof.decode_max`` / ``proof.sparse_topk``), with the true / base sets given per row as
CSR (``ptr [B + 1]``, ids).  Integer work only, so results are exact: memberships by sorted
key search, first occurrences by a stable key sort, prefix sums along the row, and the
tie-breaks as successive masked maxima / minima over the cuts.
"""
from __future__ import annotations

import torch


def _row_ids(ptr: torch.Tensor) -> torch.Tensor:
    counts = (ptr[1:] - ptr[:-1]).long()
    return torch.repeat_interleave(torch.arange(counts.numel(), device=ptr.device), counts)


def best_k_rows(tails: torch.Tensor, counts: torch.Tensor, true_ptr: torch.Tensor, true_ids: torch.Tensor,
                base_ptr: torch.Tensor, base_ids: torch.Tensor):
    """Per row: (best k, wrong at k, new at k, new true at k) as int64 [B] tensors."""
    dev = tails.device
    B, K = (int(s) for s in tails.shape)
    tails = tails.long()
    counts = counts.long().to(dev)
    pos = torch.arange(K, device=dev)
    valid = pos[None, :] < counts[:, None]
    true_ids = true_ids.long().to(dev)
    base_ids = base_ids.long().to(dev)
    span = int(max([1] + [int(x.max()) + 1 for x in (tails, true_ids, base_ids) if x.numel()]))
    rows = torch.arange(B, device=dev)[:, None]
    cand = rows * span + tails.clamp_min(0)
    true_keys = _row_ids(true_ptr.to(dev)) * span + true_ids
    base_keys = _row_ids(base_ptr.to(dev)) * span + base_ids
    in_true = torch.isin(cand, true_keys) & valid
    not_base = ~torch.isin(cand, base_keys) & valid
    # first occurrence of each tail inside its row (array order)
    flat = torch.where(valid, cand, torch.full_like(cand, -1)).reshape(-1)
    order = torch.sort(flat, stable=True).indices
    sk = flat[order]
    head = torch.ones_like(sk, dtype=torch.bool)
    head[1:] = sk[1:] != sk[:-1]
    first = torch.zeros_like(flat, dtype=torch.bool)
    first[order[head]] = True
    first = first.reshape(B, K) & valid
    # base ids that are true, per row (duplicated base ids count each time)
    base_rows = _row_ids(base_ptr.to(dev))
    base_true = torch.zeros(B, dtype=torch.int64, device=dev).index_add_(
        0, base_rows, torch.isin(base_keys, true_keys).long())
    n_true = (true_ptr[1:] - true_ptr[:-1]).long().to(dev)

    def prefix(m):
        return torch.cat([torch.zeros(B, 1, dtype=torch.int64, device=dev), torch.cumsum(m.long(), dim=1)], dim=1)

    pn, pt = prefix(not_base), prefix(not_base & in_true)
    true_count = base_true[:, None] + pt
    wrong = pn - pt
    gain = true_count - wrong
    # over the cuts k <= count: max gain, then max true count, then min wrong, then the first k
    ks = torch.arange(K + 1, device=dev)[None, :]
    ok = ks <= counts[:, None]
    big = torch.iinfo(torch.int64).max
    small = torch.iinfo(torch.int64).min
    m = ok & (gain == torch.where(ok, gain, small).max(dim=1, keepdim=True).values)
    m &= true_count == torch.where(m, true_count, small).max(dim=1, keepdim=True).values
    m &= wrong == torch.where(m, wrong, big).min(dim=1, keepdim=True).values
    best = torch.argmax(m.to(torch.int8), dim=1)
    best = torch.where((counts == 0) | (n_true == 0), torch.zeros_like(best), best)
    cn, cnt = prefix(first & not_base), prefix(first & not_base & in_true)
    g = best[:, None]
    w = torch.gather(wrong, 1, g)[:, 0]
    w = torch.where((counts == 0) | (n_true == 0), torch.zeros_like(w), w)
    return best, w, torch.gather(cn, 1, g)[:, 0], torch.gather(cnt, 1, g)[:, 0]


class DecodeAccumulator:
    """Batched ``_OracleRelationAccumulator`` (decode.py:72-150) with device counters."""

    def __init__(self, device="cuda"):
        self.device = torch.device(device)
        self._c = torch.zeros(7, dtype=torch.int64, device=self.device)

    def add_rows(self, tails, counts, true_ptr, true_ids, base_ptr, base_ids) -> torch.Tensor:
        best, wrong, new, new_true = best_k_rows(tails, counts, true_ptr, true_ids, base_ptr, base_ids)
        counts = counts.long().to(self.device)
        upd = torch.stack([counts.sum(), counts.max() if counts.numel() else counts.sum(), (best > 0).sum(),
                           best.sum(), wrong.sum(), new.sum(), new_true.sum()])
        self._c[0] += upd[0]
        self._c[1] = torch.maximum(self._c[1], upd[1])
        self._c[2:] += upd[2:]
        return best

    @property
    def counters(self) -> list[int]:
        """[candidate_total, max_candidate_count, query_count, selected, selected_wrong, new, new_true]"""
        return [int(x) for x in self._c.tolist()]

    def row(self, relation: int, truth_count: int, supply_count: int, queries: int) -> dict:
        """The per-relation summary of decode.py:118-150."""
        cand, _mx, _q, sel, sel_wrong, new, new_true = self.counters
        return {"relation": int(relation), "facts": int(truth_count), "supply": int(supply_count),
                "generated": int(supply_count + new), "missing": int(truth_count - supply_count - new_true),
                "extra": int(new - new_true), "queries": int(queries), "candidates": int(cand),
                "selected": int(sel), "selected_wrong": int(sel_wrong)}
