"""Query planning around the hop loop: the training batch split and first-hop query pruning.

* ``tnb_batch_plan`` — the training batch split (tnb_batching.py:6-20); it only sets the
  batch size B the hop loop runs at (train.py:199-203).
* ``prepare_rule_first_hop_prune`` / ``rule_first_hop_query_heads`` — the "rule_first_hop"
  decode pruning (decode_core.py:287-348): a query head is kept only if it has a supplied
  fact in some channel whose first-hop rule weight, maximised over rules, reaches
  ``args.decode_query_rule_threshold``.  The per-channel endpoint sets are built with torch
  on the device the facts live on (a whole-graph pass of gathers and ``unique``), instead
  of the reference's 5M-row numpy chunks; the results are the same sorted entity sets.
* ``first_hop_supported_entities`` — the same test as a dense bool [E] mask over a
  resident ``DeviceGraph`` (per-fact endpoints from the native fact table), for callers
  that filter device-resident query heads without a host round trip.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from . import rules


@dataclass(frozen=True)
class TnbBatchPlan:
    true_target_batch_size: int
    false_main_batch_count: int


def tnb_batch_plan(args, nominal_batch_size: int) -> TnbBatchPlan:
    """True-target and false-main batch sizes for a nominal batch (tnb_batching.py:12-20)."""
    nominal = max(1, int(nominal_batch_size))
    false_count = 0 if args.dataset == "family" else min(nominal - 1, int(round(nominal * 0.5)))
    return TnbBatchPlan(true_target_batch_size=max(1, nominal - false_count), false_main_batch_count=false_count)


def rule_first_hop_channels(weights: torch.Tensor, threshold: float) -> torch.Tensor:
    """Channels whose first-hop weight, maximised over rules, reaches ``threshold``.

    ``weights`` is the softmax of one relation's first-hop rule logits, [L, n] or [1, L, n]
    (decode_core.py:302-307).  Returns the int64 channel ids in ascending order."""
    w = weights.reshape(-1, weights.shape[-1])
    return torch.nonzero(w.amax(dim=0) >= threshold, as_tuple=False).reshape(-1)


def _facts_tensor(facts) -> torch.Tensor:
    if isinstance(facts, torch.Tensor):
        return facts
    return torch.from_numpy(np.ascontiguousarray(np.asarray(facts, dtype=np.int64)))


def prepare_rule_first_hop_prune(model, relations: Sequence[int], facts, hard_supply_np, args) -> None:
    """Per-relation active channels and per-channel supported endpoints (decode_core.py:287-331).

    Same arguments and effect as the reference: with ``args.decode_query_prune ==
    "rule_first_hop"`` and a positive ``args.decode_query_rule_threshold`` it stores
    ``args._decode_query_active_channels`` (relation -> list of channel ids) and
    ``args._decode_query_channel_heads`` (channel -> sorted int64 entity ids: the heads of
    the supplied facts of relation c for channel c, their tails for channel c + R).
    ``facts`` is [T, 3] (head, relation, tail), numpy or torch; ``hard_supply_np`` is bool [T].
    """
    if str(getattr(args, "decode_query_prune", "none")) != "rule_first_hop":
        return
    threshold = float(getattr(args, "decode_query_rule_threshold", 0.0))
    if threshold <= 0.0:
        return
    R = int(model.relation_count)
    active_by_relation: dict[int, list[int]] = {}
    with torch.no_grad():
        if rules.has_lstm_producer(model) and model.emb.is_cuda and len(relations):
            # every relation at once through the device producer: hop-0 weights [U, L, n]
            w0 = rules.rule_weights(model, torch.tensor([int(r) for r in relations], device=model.emb.device))[0]
            for i, relation in enumerate(relations):
                active_by_relation[int(relation)] = rule_first_hop_channels(w0[i:i + 1], threshold).cpu().tolist()
        else:
            for relation in relations:
                logits = model.build_rule_logits(torch.tensor([relation], device=model.emb.device))
                weights = torch.softmax(logits[:, 0, :, :] / model.tau_1, dim=-1)
                active_by_relation[int(relation)] = rule_first_hop_channels(weights, threshold).cpu().tolist()
    wanted = sorted({c % R for chans in active_by_relation.values() for c in chans if c < 2 * R})
    ft = _facts_tensor(facts)
    dev = ft.device
    head, rel, tail = ft[:, 0].long(), ft[:, 1].long(), ft[:, 2].long()
    supply = torch.as_tensor(np.asarray(hard_supply_np) if not isinstance(hard_supply_np, torch.Tensor)
                             else hard_supply_np).to(dev).reshape(-1).bool()
    is_wanted = torch.zeros(R, dtype=torch.bool, device=dev)
    if wanted:
        is_wanted[torch.tensor(wanted, device=dev)] = True
    keep = supply & is_wanted[rel]
    h, r, t = head[keep], rel[keep], tail[keep]
    cache: dict[int, np.ndarray] = {}
    for relation in wanted:
        sel = r == relation
        cache[relation] = torch.unique(h[sel]).cpu().numpy().astype(np.int64)
        cache[relation + R] = torch.unique(t[sel]).cpu().numpy().astype(np.int64)
    args._decode_query_channel_heads = cache
    args._decode_query_active_channels = active_by_relation


def rule_first_hop_query_heads(relation: int, query_heads: Sequence[int], args) -> list[int]:
    """The query heads, in their given order, that some active channel supports (decode_core.py:334-347)."""
    if str(getattr(args, "decode_query_prune", "none")) != "rule_first_hop":
        return list(query_heads)
    channels = getattr(args, "_decode_query_active_channels", {}).get(int(relation), [])
    cache = getattr(args, "_decode_query_channel_heads", {})
    supported = [cache[c] for c in channels if c in cache]
    if not supported:
        return []
    heads = np.asarray(query_heads, dtype=np.int64)
    return heads[np.isin(heads, np.concatenate(supported))].tolist()


def first_hop_supported_entities(graph, channels: torch.Tensor, supply_mask: torch.Tensor | None = None
                                 ) -> torch.Tensor:
    """bool [E] on the graph's device: entities with a supplied fact in one of ``channels``.

    Channel c < R is relation c read head -> tail, so the fact's head is supported
    (``cache[c]`` above); channel R + c is relation c read tail -> head, so the fact's tail is
    supported (``cache[c + R]``).  The identity channel 2R adds nothing.  ``supply_mask``
    (bool [T], by fact id; default all facts) selects the supplied facts."""
    dev = graph.device
    E, R = graph.num_entities, graph.num_relations
    ch = channels.to(dev).long()
    want = torch.zeros(2 * R, dtype=torch.bool, device=dev)
    want[ch[(ch >= 0) & (ch < 2 * R)]] = True
    head, tail, rel = graph.fact_table()
    rel = rel.long()
    supplied = None if supply_mask is None else supply_mask.to(dev).reshape(-1).bool()
    supported = torch.zeros(E, dtype=torch.bool, device=dev)
    for endpoint, offset in ((head, 0), (tail, R)):
        keep = want[rel + offset]
        if supplied is not None:
            keep &= supplied
        supported[endpoint.long()[keep]] = True
    return supported
