"""Parity on the named workloads at their full graph sizes.

The oracle checks a few queries of each workload on the full graph; the full query batch is
then tied to those queries by per-query independence (every (query, rule) column of the hop
loop is computed independently), and checked by size-independent properties (mass bound,
finiteness, bit-exact decode rows).  kg_small / kg_mid / kg_skew run the fused loop (uncapped,
kg_skew with its 1e-4 state threshold); kg_large (cap 100) and a 2%-scale kg_web (cap 50) run
the capped hop-by-hop op, including output keys beyond 2^32.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import fastlog_oracle as O
from tests.conftest import GRAD_ATOL, GRAD_RTOL, exact_loop_grads, softmax_backward

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
RTOL, ATOL = 1e-5, 1e-6
SUB = 4  # queries checked against the oracle

_CACHE: dict = {}


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def workload(name: str):
    """(workload, kg, oracle csr, DeviceGraph, hop inputs), built once per module."""
    if name not in _CACHE:
        from minikg_dev_b200.graph import DeviceGraph
        from minikg_dev_b200.synth import WORKLOADS, hop_inputs, sample_graph, scaled_workload
        base, _, factor = name.partition("@")
        wl = scaled_workload(base, float(factor)) if factor else WORKLOADS[base]
        kg = sample_graph(wl.E, wl.R, wl.T, wl.gen, seed=0, name=wl.name)
        csr = O.build_csr_structure(kg.head, kg.tail, kg.rel, kg.num_entities)
        dg = DeviceGraph(tuple(T(a) for a in csr), kg.num_entities, kg.num_relations)
        inp = hop_inputs(kg, wl.B, wl.L, wl.hops, seed=0)
        while len(_CACHE) >= 2:  # at most two graphs resident
            _CACHE.pop(next(iter(_CACHE)))
        _CACHE[name] = (wl, kg, csr, dg, inp)
    return _CACHE[name]


def _assert_close(got, want, thr, rtol=RTOL, atol=ATOL):
    """allclose; with a state threshold, a value that lands within fp32 rounding of it may be
    kept by one summation order and dropped by another: such flips (a tiny share of entries,
    each moving the result by at most a few thresholds) are allowed."""
    if thr <= 0:
        np.testing.assert_array_equal(got != 0, want != 0)
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)
        return
    bad = ~np.isclose(got, want, rtol=rtol, atol=atol)
    assert bad.sum() <= max(2, 1e-4 * got.size), f"{bad.sum()} entries differ"
    assert np.abs(got - want)[bad].max(initial=0.0) <= 4 * thr


def _dense(keys2, vals, B, E):
    out = np.zeros((B, E), np.float32)
    out[keys2 // E, keys2 % E] = vals
    return out


FUSED = ["kg_small", "kg_mid", "kg_skew"]


@pytest.mark.parametrize("name", FUSED)
def test_fused_loop_subset_vs_oracle(name):
    from minikg_dev_b200.proof import proof_scores
    wl, kg, csr, dg, inp = workload(name)
    E, R, L, K = kg.num_entities, kg.num_relations, wl.L, wl.hops
    heads, w = inp.heads[:SUB], inp.rule_weights[:, :SUB]
    final, trace = O.proof_sum_forward(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R,
                                       threshold=wl.state_threshold)
    wt = T(w).requires_grad_(True)
    sc = T(inp.edge_scores).requires_grad_(True)
    out, msgs = proof_scores(dg, T(heads), wt, sc, mask=None, threshold=wl.state_threshold)
    want = _dense(final[0], final[1], SUB, E)
    got = out.detach().cpu().numpy()
    _assert_close(got, want, wl.state_threshold)
    exp_msgs = [O.count_messages(tr["state"], csr, w[k], L, E, R) for k, tr in enumerate(trace)]
    if wl.state_threshold > 0:
        np.testing.assert_allclose(msgs.cpu().numpy(), exp_msgs, rtol=1e-3)
    else:
        assert msgs.cpu().tolist() == exp_msgs
    seed = np.random.default_rng(3).standard_normal(final[0].shape[0]).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R, final[0], seed,
                              num_facts=kg.num_triples, threshold=wl.state_threshold)
    (out * T(_dense(final[0], seed, SUB, E))).sum().backward()
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("name", FUSED)
def test_fused_capped_subset_vs_oracle(name):
    """The reference's production edge cap (100) on the fused loop, full graph, a query subset."""
    from minikg_dev_b200.proof import proof_scores
    wl, kg, csr, dg, inp = workload(name)
    E, R, L, K = kg.num_entities, kg.num_relations, wl.L, wl.hops
    cap = 100
    heads, w = inp.heads[:SUB], inp.rule_weights[:, :SUB]
    final, trace = O.proof_sum_forward(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R, cap=cap,
                                       threshold=wl.state_threshold)
    wt = T(w).requires_grad_(True)
    sc = T(inp.edge_scores).requires_grad_(True)
    out, msgs = proof_scores(dg, T(heads), wt, sc, mask=None, threshold=wl.state_threshold, topk_edges=cap)
    _assert_close(out.detach().cpu().numpy(), _dense(final[0], final[1], SUB, E), wl.state_threshold)
    exp_msgs = [O.count_messages(tr["state"], csr, w[k], L, E, R, cap=cap) for k, tr in enumerate(trace)]
    if wl.state_threshold > 0:
        np.testing.assert_allclose(msgs.cpu().numpy(), exp_msgs, rtol=1e-3)
    else:
        assert msgs.cpu().tolist() == exp_msgs
    seed = np.random.default_rng(5).standard_normal(final[0].shape[0]).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R, final[0], seed,
                              num_facts=kg.num_triples, cap=cap, threshold=wl.state_threshold)
    (out * T(_dense(final[0], seed, SUB, E))).sum().backward()
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("name", FUSED)
def test_fused_loop_full_batch(name):
    """Full B: the first queries match the oracle-checked subset run; per-query mass <= L; the
    full batch's rule-weight gradient of the first queries (queries are independent) is held to
    the bar against the oracle's float64 run of those queries."""
    from minikg_dev_b200.proof import proof_scores
    wl, kg, csr, dg, inp = workload(name)
    E, R, B, L = kg.num_entities, kg.num_relations, wl.B, wl.L
    sc = T(inp.edge_scores)
    wt = T(inp.rule_weights).requires_grad_(True)
    out, msgs = proof_scores(dg, T(inp.heads), wt, sc, mask=None, threshold=wl.state_threshold)
    seed = torch.randn(B, E, device=DEV, generator=torch.Generator(DEV).manual_seed(1)) * (out != 0)
    (out * seed).sum().backward()
    sub, _ = proof_scores(dg, T(inp.heads[:SUB]), T(inp.rule_weights[:, :SUB]), sc, mask=None,
                          threshold=wl.state_threshold)
    full = out.detach()
    assert torch.isfinite(full).all() and (full >= 0).all()
    assert (full.sum(dim=1) <= L * (1 + 1e-5)).all()
    _assert_close(full[:SUB].cpu().numpy(), sub.detach().cpu().numpy(), wl.state_threshold)
    heads, w = inp.heads[:SUB], inp.rule_weights[:, :SUB]
    final, _ = O.proof_sum_forward(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R,
                                   threshold=wl.state_threshold)
    s_np = seed[:SUB].cpu().numpy().reshape(-1)[final[0]]
    gw, _ = exact_loop_grads(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R, final[0], s_np,
                             num_facts=kg.num_triples, threshold=wl.state_threshold)
    np.testing.assert_allclose(wt.grad[:, :SUB].cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    assert int(msgs.sum()) > 0


@pytest.mark.parametrize("name", FUSED)
def test_max_decode_full_batch_vs_oracle(name):
    """Full-B max decode (top-100): the first queries bit-exact against the oracle."""
    from minikg_dev_b200.proof import decode_max
    wl, kg, csr, dg, inp = workload(name)
    E, R, L = kg.num_entities, kg.num_relations, wl.L
    res = decode_max(dg, T(inp.heads), T(inp.rule_weights), 100, T(inp.edge_scores))
    final, _ = O.proof_max_forward(inp.heads[:SUB], inp.rule_weights[:, :SUB], csr, inp.edge_mask, inp.edge_scores,
                                   SUB, L, E, R)
    np.testing.assert_array_equal(res.raw[:SUB].cpu().numpy(), _dense(final[0], final[1], SUB, E))
    ot, osc, oc = O.decode_topk(final, SUB, E, 100)
    np.testing.assert_array_equal(res.tails[:SUB].cpu().numpy(), ot)
    np.testing.assert_array_equal(res.scores[:SUB].cpu().numpy(), osc)
    np.testing.assert_array_equal(res.counts[:SUB].cpu().numpy(), oc)
    assert (res.counts.cpu().numpy() <= 100).all()


# ----------------------------------------------------------------------------- capped, large graphs
CAPPED = ["kg_large", "kg_web@0.02"]


def _duck(kg, wl, logits, scores_t, cap, topk_nodes):
    """The model / graph / args surface kernel_sparse_scores reads (proof.py:467-614); the
    CSR is built from the triples on the device, as on the reference's first call."""
    K, B, L, n = logits.shape
    lg = logits.permute(1, 0, 2, 3)  # [B, K, L, n]
    model = SimpleNamespace(rules=L, entity_count=kg.num_entities, relation_count=kg.num_relations, step=K,
                            tau_1=1.0, weight=scores_t, dropout=torch.nn.Identity(),
                            build_rule_logits=lambda rels: lg)
    mask = torch.ones(kg.num_triples, dtype=torch.bool, device=DEV)
    graph = SimpleNamespace(e2triple=(T(kg.head), None, mask), triple2e=(None, T(kg.tail), mask),
                            r2triple=(T(kg.rel), None, mask), mask=mask, mask_float=mask.float())
    args = SimpleNamespace(kernel_topk_edges=cap, kernel_topk_nodes=topk_nodes)
    return model, graph, args


def test_first_hop_pruned_max_decode_kg_large():
    """kg_large's decode: first-hop query pruning (decode_core.py:287-348) on the device graph,
    then the capped max decode of the surviving heads, against the oracle on the same heads."""
    from minikg_dev_b200.batching import first_hop_supported_entities, rule_first_hop_channels
    from minikg_dev_b200.proof import decode_max_sparse
    wl, kg, csr, dg, inp = workload("kg_large")
    E, R, L = kg.num_entities, kg.num_relations, wl.L
    rng = np.random.default_rng(23)
    n = 2 * R + 1
    logits = (rng.standard_normal((L, n)) * 3.0).astype(np.float32)  # one relation's first-hop rule logits
    chans = rule_first_hop_channels(torch.softmax(torch.from_numpy(logits), dim=-1), 0.2)
    assert chans.numel() > 0
    supported = first_hop_supported_entities(dg, chans)
    cand = T(rng.integers(0, E, 64).astype(np.int64))
    kept = cand[supported[cand]]
    # oracle restatement of the same pruning
    chans_np = chans.numpy()
    cache = O.rule_first_hop_cache(kg.head, kg.rel, kg.tail, np.ones(kg.num_triples, bool),
                                   sorted({int(c) % R for c in chans_np if c < 2 * R}), R)
    want_kept = O.rule_first_hop_query_heads(chans_np, cache, cand.cpu().numpy())
    np.testing.assert_array_equal(kept.cpu().numpy(), want_kept)
    Bk = int(kept.numel())
    if Bk == 0:
        return
    w = inp.rule_weights[:, :1].repeat(Bk, axis=1)
    final, tails, sc, counts = decode_max_sparse(dg, kept, T(w), 100, T(inp.edge_scores), cap=wl.capped_row)
    want, _ = O.proof_max_forward(kept.cpu().numpy(), w, csr, inp.edge_mask, inp.edge_scores, Bk, L, E, R,
                                  cap=wl.capped_row)
    idx = final.indices().cpu().numpy()
    np.testing.assert_array_equal(idx[0] * E + idx[1], want[0])
    np.testing.assert_array_equal(final.values().cpu().numpy(), want[1])
    ot, osc, _ = O.decode_topk(want, Bk, E, 100)
    np.testing.assert_array_equal(tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(sc.cpu().numpy(), osc)


@pytest.mark.parametrize("name", ["kg_large", "kg_web@0.02"])
def test_capped_max_decode_subset_vs_oracle(name):
    """The capped hop-by-hop max decode (the large graphs' decode path) bit-exact on a query subset."""
    from minikg_dev_b200.proof import decode_max_sparse
    wl, kg, csr, dg, inp = workload(name)
    E, R, L = kg.num_entities, kg.num_relations, wl.L
    w = inp.rule_weights[:, :SUB]
    final, tails, sc, counts = decode_max_sparse(dg, T(inp.heads[:SUB]), T(w), 100, T(inp.edge_scores),
                                                 cap=wl.capped_row)
    want, _ = O.proof_max_forward(inp.heads[:SUB], w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R,
                                  cap=wl.capped_row)
    idx = final.indices().cpu().numpy()
    np.testing.assert_array_equal(idx[0] * E + idx[1], want[0])
    np.testing.assert_array_equal(final.values().cpu().numpy(), want[1])
    ot, osc, oc = O.decode_topk(want, SUB, E, 100)
    np.testing.assert_array_equal(tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(sc.cpu().numpy(), osc)
    np.testing.assert_array_equal(counts.cpu().numpy(), oc)


def test_hop_op_keys_beyond_32_bits():
    """kg_large at its full B x L: output keys b*L*E + l*E + e exceed 2^32 (256 x 4 x 4.59M)."""
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    wl, kg, csr, dg, inp = workload("kg_large")
    E, R, B, L = kg.num_entities, kg.num_relations, wl.B, wl.L
    assert B * L * E > 2 ** 32
    rng = np.random.default_rng(11)
    rows = [(b, l) for b in (0, 100, B - 2, B - 1) for l in range(L)]
    deg = np.bincount(kg.head, minlength=E) + np.bincount(kg.tail, minlength=E)
    ents = np.concatenate([np.argsort(-deg)[:4], rng.integers(0, E, 12)])
    keys = np.unique(np.array([(b * L + l) * E + e for b, l in rows for e in ents], np.int64))
    fb, fl, fe = O.split3(keys, L, E)
    fv = rng.uniform(0.05, 1.0, keys.shape[0]).astype(np.float32)
    w = inp.rule_weights[0]
    fwd = O.sparse3d_forward(fb, fl, fe, fv, w, csr, inp.edge_mask, inp.edge_scores, B, L, E, R, cap=wl.capped_row,
                             agg_mode=0, is_score=True)
    o, i, d = FastLogFunctionSparse3DTopK.apply(T(fb), T(fl), T(fe), T(fv), T(w), *dg.csr,
                                                torch.ones((), device=DEV), T(inp.edge_scores), B, L, E, R, False,
                                                wl.capped_row, 0, True, 1.0)
    for name, t in (("ori", o), ("inv", i), ("ind", d)):
        t = t.coalesce()
        idx = t.indices().cpu().numpy()
        got = O.keys3(idx[0], idx[1], idx[2], L, E)
        np.testing.assert_array_equal(got, fwd[name][0], err_msg=name)
        np.testing.assert_allclose(t.values().cpu().numpy(), fwd[name][1], rtol=RTOL, atol=ATOL, err_msg=name)
    assert fwd["ori"][0].max() > 2 ** 32


@pytest.mark.parametrize("name", CAPPED)
@pytest.mark.parametrize("capped", [False, True])
def test_large_graph_hops_subset_vs_oracle(name, capped):
    """kernel_sparse_scores on the full large graphs, a query subset: uncapped with the
    workload's frontier prune (the key-slab loop) and with the production edge cap (the sparse
    loop); keys exact, values and gradients at the bar."""
    from minikg_dev_b200.proof import kernel_sparse_scores
    wl, kg, csr, dg, inp = workload(name)
    E, R, L, K = kg.num_entities, kg.num_relations, wl.L, wl.hops
    cap = wl.capped_row if capped else wl.topk_edges
    heads = inp.heads[:SUB]
    logits = T(inp.rule_logits[:, :SUB]).requires_grad_(True)
    sc = T(inp.edge_scores).requires_grad_(True)
    model, graph, args = _duck(kg, wl, logits, sc, cap, wl.topk_nodes)
    out = kernel_sparse_scores(model, T(heads), T(np.zeros(SUB, np.int64)), graph, args, is_training=True).coalesce()
    # the oracle gets the device's own softmax: a one-ulp weight difference can move a cap bucket
    w = torch.softmax(logits.detach(), dim=-1).cpu().numpy()
    final, trace = O.proof_sum_forward(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R,
                                       cap=cap, topk_nodes=wl.topk_nodes)
    idx = out.indices().cpu().numpy()
    np.testing.assert_array_equal(idx[0] * E + idx[1], final[0])
    np.testing.assert_allclose(out.values().detach().cpu().numpy(), final[1], rtol=RTOL, atol=ATOL)
    seed = np.random.default_rng(5).standard_normal(final[0].shape[0]).astype(np.float32)
    (out.values() * T(seed)).sum().backward()
    gw, ge = exact_loop_grads(heads, w, csr, inp.edge_mask, inp.edge_scores, SUB, L, E, R, final[0], seed,
                              num_facts=kg.num_triples, cap=cap, topk_nodes=wl.topk_nodes)
    np.testing.assert_allclose(logits.grad.cpu().numpy(), softmax_backward(w, gw), rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


def test_slab_loop_full_batch_kg_large():
    """The uncapped 4.59M-entity loop at its full batch (256 queries x 4 rules, 2 hops): the
    first queries equal the oracle-checked subset run (the frontier prune at 0.5% of the
    entities does not cut the hop-1 frontier, so queries stay independent), every value is
    finite and positive, each query's mass is at most L, and the message count is the sum of
    the frontier's out-degrees."""
    from minikg_dev_b200.slab_loop import slab_engine, slab_proof_scores
    wl, kg, csr, dg, inp = workload("kg_large")
    E, B, L = kg.num_entities, wl.B, wl.L
    eng = slab_engine(dg)
    sc = T(inp.edge_scores).requires_grad_(True)
    wt = T(inp.rule_weights).requires_grad_(True)
    out, msgs = slab_proof_scores(eng, T(inp.heads), wt, sc, None, True, 1.0, wl.topk_nodes)
    out = out.coalesce()
    vals = out.values()
    assert torch.isfinite(vals).all() and (vals > 0).all()
    per_q = torch.zeros(B, device=DEV).index_add_(0, out.indices()[0], vals.detach())
    assert (per_q <= L * (1 + 1e-5)).all()
    seed = torch.randn(vals.numel(), device=DEV, generator=torch.Generator(DEV).manual_seed(4))
    (vals * seed).sum().backward()
    sub, _ = slab_proof_scores(eng, T(inp.heads[:SUB]), T(inp.rule_weights[:, :SUB]), sc.detach(), None, True, 1.0,
                               wl.topk_nodes)
    sub = sub.coalesce()
    first = out.indices()[0] < SUB
    assert torch.equal(out.indices()[:, first], sub.indices())
    np.testing.assert_allclose(vals.detach()[first].cpu().numpy(), sub.values().detach().cpu().numpy(), rtol=RTOL,
                               atol=ATOL)
    # the full batch's gradient of the first queries against the oracle's float64 run of them
    si = sub.indices().cpu().numpy()
    gw, _ = exact_loop_grads(inp.heads[:SUB], inp.rule_weights[:, :SUB], csr, inp.edge_mask, inp.edge_scores, SUB,
                             L, E, kg.num_relations, si[0] * E + si[1], seed[first].cpu().numpy(),
                             num_facts=kg.num_triples, topk_nodes=wl.topk_nodes)
    np.testing.assert_allclose(wt.grad[:, :SUB].cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    assert int(msgs[0]) == int(dg.push_degree()[T(inp.heads)].sum()) * L
    assert int(msgs.sum()) > 10_000_000
