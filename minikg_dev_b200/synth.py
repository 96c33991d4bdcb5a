"""Seeded synthetic knowledge graphs and hop inputs.

The graphs stand in for the datasets the reference trains on (family, CoDEx-M,
YAGO3-10, Wikidata5M, Freebase): same entity / relation / triple counts and the
stated skew, drawn from a seeded ``numpy.random.default_rng``.  None of the
datasets' own records are used.

A graph is a ``KG`` with int32 ``head``, ``rel``, ``tail`` arrays of length T
(unique (head, rel, tail) triples, in sampling order) plus its entity and
relation counts.  ``hop_inputs`` draws the per-query inputs the hop loop needs:
query heads (uniform), per-hop rule weights ``softmax(N(0,1))`` over the
n = 2R+1 channels, and per-fact edge scores in (0, 1].
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class KG:
    name: str
    num_entities: int
    num_relations: int
    head: np.ndarray
    rel: np.ndarray
    tail: np.ndarray
    meta: dict = field(default_factory=dict)

    @property
    def num_triples(self) -> int:
        return int(self.head.shape[0])


@dataclass(frozen=True)
class Workload:
    """One benchmark / parity configuration: a graph shape plus the hop-loop shape."""
    name: str
    E: int
    R: int
    T: int
    B: int
    L: int
    hops: int
    topk_edges: int = 1 << 60
    topk_nodes: int = 0
    state_threshold: float = 0.0  # harness rule: drop state values below this after each hop
    gen: tuple = ()               # generator knobs, see _sample_graph
    note: str = ""
    capped_row: int = 1 << 60     # the reference's production edge cap for this dataset shape


UNCAPPED = 1 << 60

# Shapes of the five reference workloads.  ``gen`` knobs:
#   rel=("zipf", s) | ("top2", share, s) | ("zipf_prefix", s, coverage)
#   head/tail=(exponent, offset) rank-frequency power laws; hubs=(frac, share)
WORKLOADS = {
    "kg_small": Workload(
        "kg_small", E=3007, R=12, T=28356, B=64, L=3, hops=3,
        gen=(("rel", ("zipf", 1.1)), ("head", (1.5, 6.0)), ("tail", (0.6, 1.0))),
        note="3,007 entities / 12 relations / 28,356 triples; relation Zipf 1.1, out-degree Zipf 1.5"),
    "kg_mid": Workload(
        "kg_mid", E=17050, R=51, T=206205, B=256, L=3, hops=3,
        gen=(("rel", ("zipf", 1.0)), ("head", (1 / 1.1, 2.0)), ("tail", (1 / 1.1, 2.0)),
             ("hubs", (0.05, 0.40))), capped_row=100,
        note="17,050 entities / 51 relations / 206,205 triples; relation Zipf 1.0, degree power law 2.1, "
             "5% hub entities receive 40% of edges"),
    "kg_skew": Workload(
        "kg_skew", E=123182, R=37, T=1089040, B=512, L=3, hops=3, state_threshold=1e-4, capped_row=100,
        gen=(("rel", ("top2", 0.70, 1.0)), ("head", (0.8, 2.0)), ("tail", (1.3, "max:50000"))),
        note="123,182 entities / 37 relations / 1,089,040 triples; top-2 relations hold 70%, "
             "in-degree Zipf 1.3 with max in-degree ~50k; state threshold 1e-4"),
    # frontier bound: the reference's entity prune (drum.py:54-80) at 0.5% of the entities
    "kg_large": Workload(
        "kg_large", E=4594485, R=822, T=20624575, B=256, L=4, hops=2, topk_nodes=22972, capped_row=100,
        gen=(("rel", ("zipf_prefix", 1.2, 0.70)), ("head", (1.0, 10.0)), ("tail", (1.0, 10.0))),
        note="4,594,485 entities / 822 relations / 20,624,575 triples; relation Zipf 1.2 truncated "
             "to the 70% prefix, degree power law 2.0; uncapped, frontier pruned to <= 0.5% of the "
             "entities (22,972)"),
    # frontier bound: the entity prune at 1M entities (<= 1M nonzeros per query and rule)
    "kg_web": Workload(
        "kg_web", E=86054151, R=14824, T=338586276, B=128, L=4, hops=2, topk_nodes=1000000, capped_row=50,
        gen=(("rel", ("zipf_prefix", 1.3, 0.80)), ("head", (1.0, 10.0)), ("tail", (1 / 0.9, "max:1000000"))),
        note="86,054,151 entities / 14,824 relations / 338,586,276 triples; relation Zipf 1.3 "
             "truncated to the 80% prefix, in-degree power law 1.9, max hub ~1M; uncapped, frontier "
             "pruned to 1M entities"),
}


def _rank_weights(n: int, exponent: float, offset, total: int, rng) -> np.ndarray:
    """Power-law weights over a random permutation of ``n`` ids.

    ``offset`` shifts the ranks (weight ∝ (rank + offset)^-exponent).  The form
    ``"max:K"`` picks the offset so the top id expects about K of ``total`` draws.
    """
    ranks = np.arange(n, dtype=np.float64)
    if isinstance(offset, str) and offset.startswith("max:"):
        target = float(offset[4:]) / float(total)
        lo, hi = 1e-3, float(n)
        for _ in range(80):  # bisection on the offset: top share falls as offset grows
            mid = np.sqrt(lo * hi)
            wts = (ranks + mid) ** (-exponent)
            share = wts[0] / wts.sum()
            if share > target:
                lo = mid
            else:
                hi = mid
        off = np.sqrt(lo * hi)
    else:
        off = float(offset)
    wts = (ranks + off) ** (-exponent)
    wts /= wts.sum()
    perm = rng.permutation(n)
    out = np.empty(n, dtype=np.float64)
    out[perm] = wts
    return out


def _relation_probs(R: int, spec, rng) -> np.ndarray:
    kind = spec[0]
    if kind == "zipf":
        p = (np.arange(R, dtype=np.float64) + 1.0) ** (-spec[1])
    elif kind == "top2":
        share, s = spec[1], spec[2]
        rest = (np.arange(R - 2, dtype=np.float64) + 1.0) ** (-s)
        rest = rest / rest.sum() * (1.0 - share)
        p = np.concatenate([[share / 2, share / 2], rest])
    elif kind == "zipf_prefix":
        s, coverage = spec[1], spec[2]
        p = (np.arange(R, dtype=np.float64) + 1.0) ** (-s)
        p /= p.sum()
        keep = int(np.searchsorted(np.cumsum(p), coverage) + 1)
        p[keep:] = 0.0
    else:
        raise ValueError(f"unknown relation spec {spec!r}")
    p = p / p.sum()
    # relation ids are a random relabelling of the frequency ranks
    perm = rng.permutation(R)
    out = np.empty(R, dtype=np.float64)
    out[perm] = p
    return out


def _draw(probs: np.ndarray, count: int, rng) -> np.ndarray:
    cdf = np.cumsum(probs)
    cdf /= cdf[-1]
    u = rng.random(count)
    if probs.shape[0] > 65536 and count > 65536:
        # same result; sorted queries keep the binary searches cache-resident on large CDFs
        order = np.argsort(u, kind="stable")
        idx = np.empty(count, dtype=np.int64)
        idx[order] = np.searchsorted(cdf, u[order], side="right")
    else:
        idx = np.searchsorted(cdf, u, side="right")
    return np.minimum(idx, probs.shape[0] - 1)


def sample_graph(E: int, R: int, T: int, gen, seed: int = 0, name: str = "kg") -> KG:
    """Draw exactly ``T`` unique (head, rel, tail) triples with the requested skew."""
    knobs = dict(gen)
    rng = np.random.default_rng(seed)
    p_rel = _relation_probs(R, knobs.get("rel", ("zipf", 1.0)), rng)
    h_exp, h_off = knobs.get("head", (1.0, 1.0))
    t_exp, t_off = knobs.get("tail", (1.0, 1.0))
    p_head = _rank_weights(E, h_exp, h_off, T, rng)
    p_tail = _rank_weights(E, t_exp, t_off, T, rng)
    hubs = knobs.get("hubs")
    hub_ids = None
    if hubs is not None:
        hub_ids = rng.choice(E, size=max(1, int(round(hubs[0] * E))), replace=False)
    if T > E * E * R:
        raise ValueError("more triples requested than distinct (head, rel, tail) combinations")

    keys_seen = np.empty(0, dtype=np.int64)
    chunks_h, chunks_r, chunks_t = [], [], []
    have = 0
    stride_t = np.int64(E)
    stride_r = np.int64(R)
    while have < T:
        need = T - have
        draw = int(need * 1.3) + 1024
        h = _draw(p_head, draw, rng)
        r = _draw(p_rel, draw, rng)
        t = _draw(p_tail, draw, rng)
        if hub_ids is not None:
            to_hub = rng.random(draw) < hubs[1]
            t = np.where(to_hub, hub_ids[rng.integers(0, hub_ids.shape[0], draw)], t)
        key = (h.astype(np.int64) * stride_r + r) * stride_t + t
        # first occurrence of each new key, in draw order
        _, first = np.unique(key, return_index=True)
        first.sort()
        key, h, r, t = key[first], h[first], r[first], t[first]
        fresh = ~np.isin(key, keys_seen, assume_unique=False)
        key, h, r, t = key[fresh], h[fresh], r[fresh], t[fresh]
        take = min(need, key.shape[0])
        chunks_h.append(h[:take]); chunks_r.append(r[:take]); chunks_t.append(t[:take])
        keys_seen = np.concatenate([keys_seen, key[:take]])
        have += take
    head = np.concatenate(chunks_h).astype(np.int32)
    rel = np.concatenate(chunks_r).astype(np.int32)
    tail = np.concatenate(chunks_t).astype(np.int32)
    return KG(name, E, R, head, rel, tail, meta={"seed": seed, "gen": gen})


def sample_graph_device(E: int, R: int, T: int, gen, seed: int = 0, device="cuda"):
    """``T`` unique (head, rel, tail) triples drawn on the GPU with the skew recipe of
    ``sample_graph`` (same rank-frequency weights, drawn with the device's Philox stream, so the
    realisation differs from ``sample_graph``'s), for graphs whose host generation would take
    minutes.  Duplicates are removed on the pair (h * R + r, t) -- no 64-bit key overflow at
    86 M entities x 14,824 relations -- keeping the first draw.  Every GPU given the same seed
    produces the same graph.  Returns int32 device tensors (head, rel, tail)."""
    import torch
    knobs = dict(gen)
    rng = np.random.default_rng(seed)
    p_rel = _relation_probs(R, knobs.get("rel", ("zipf", 1.0)), rng)
    h_exp, h_off = knobs.get("head", (1.0, 1.0))
    t_exp, t_off = knobs.get("tail", (1.0, 1.0))
    cdfs = []
    for p in (_rank_weights(E, h_exp, h_off, T, rng), p_rel, _rank_weights(E, t_exp, t_off, T, rng)):
        c = torch.from_numpy(np.cumsum(p)).to(device)
        cdfs.append(c / c[-1])
    if knobs.get("hubs") is not None:
        raise ValueError("sample_graph_device: hub redirection is not supported")
    gdev = torch.Generator(device=device).manual_seed(int(seed))
    k1 = torch.empty(0, dtype=torch.int64, device=device)
    k2 = torch.empty(0, dtype=torch.int64, device=device)
    while k1.numel() < T:
        need = T - k1.numel()
        draw = int(need * 1.3) + 1024
        idx = []
        for c in cdfs:
            u = torch.rand(draw, dtype=torch.float64, device=device, generator=gdev)
            idx.append(torch.clamp(torch.searchsorted(c, u, right=True), max=c.numel() - 1))
        h, r, t = idx
        n1 = torch.cat([k1, h * R + r])
        n2 = torch.cat([k2, t])
        order = torch.arange(n1.numel(), device=device)
        o = torch.sort(n2, stable=True).indices
        o = o[torch.sort(n1[o], stable=True).indices]  # (k1, k2) ascending, draw order inside ties
        first = torch.ones(o.numel(), dtype=torch.bool, device=device)
        first[1:] = (n1[o][1:] != n1[o][:-1]) | (n2[o][1:] != n2[o][:-1])
        keep = torch.sort(order[o][first]).values       # first occurrences, in draw order
        fresh = keep[keep >= k1.numel()][:need]
        k1 = torch.cat([k1, n1[fresh]])
        k2 = torch.cat([k2, n2[fresh]])
        del n1, n2, order, o, first, keep, idx, h, r, t
    return (k1 // R).to(torch.int32), (k1 % R).to(torch.int32), k2.to(torch.int32)


def workload_graph(name: str, seed: int = 0) -> KG:
    wl = WORKLOADS[name]
    return sample_graph(wl.E, wl.R, wl.T, wl.gen, seed=seed, name=name)


def scaled_workload(name: str, factor: float) -> Workload:
    """The same skew recipe at ``factor`` of the entity / triple counts (parity-sized cases)."""
    wl = WORKLOADS[name]
    E = max(64, int(wl.E * factor))
    T = max(256, int(wl.T * factor))
    gen = tuple((k, v) if not (k in ("head", "tail") and isinstance(v[1], str))
                else (k, (v[0], "max:%d" % max(8, int(float(v[1][4:]) * factor)))) for k, v in wl.gen)
    return Workload(f"{name}@{factor:g}", E=E, R=wl.R, T=T, B=wl.B, L=wl.L, hops=wl.hops,
                    topk_edges=wl.topk_edges, topk_nodes=int(wl.topk_nodes * factor) if wl.topk_nodes else 0,
                    state_threshold=wl.state_threshold, gen=gen, note=wl.note + f" (scaled x{factor:g})",
                    capped_row=wl.capped_row)


@dataclass
class HopInputs:
    heads: np.ndarray        # int64 [B]
    rule_logits: np.ndarray  # float32 [hops, B, L, n]
    rule_weights: np.ndarray # float32 [hops, B, L, n] = softmax(rule_logits) over n
    edge_scores: np.ndarray  # float32 [T] in (0, 1]
    edge_mask: np.ndarray    # bool [T]


def softmax_f32(x: np.ndarray, axis: int = -1) -> np.ndarray:
    x = x.astype(np.float64)
    x = x - x.max(axis=axis, keepdims=True)
    e = np.exp(x)
    return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)


def hop_inputs(kg: KG, B: int, L: int, hops: int, seed: int = 0,
               mask_false_frac: float = 0.0) -> HopInputs:
    rng = np.random.default_rng(seed + 1)
    n = 2 * kg.num_relations + 1
    heads = rng.integers(0, kg.num_entities, size=B).astype(np.int64)
    logits = rng.standard_normal((hops, B, L, n)).astype(np.float32)
    weights = softmax_f32(logits, axis=-1)
    scores = (1.0 / (1.0 + np.exp(-rng.standard_normal(kg.num_triples) * 1.5))).astype(np.float32)
    scores = np.maximum(scores, np.float32(1e-3))
    mask = np.ones(kg.num_triples, dtype=bool)
    if mask_false_frac > 0:
        mask &= rng.random(kg.num_triples) >= mask_false_frac
    return HopInputs(heads, logits, weights, scores, mask)
