"""Destination ranges of the CUDA hop op and the sharded loop over NCCL.

* one GPU: the outputs of ``HopRange`` over a partition of [0, E) are exactly the full-range
  op's outputs split by destination, and their gradients add up to the full-range ones;
* two GPUs (skipped with fewer): the destination-partitioned loop (one process per GPU,
  NCCL) against the single-process oracle on a 2%-scale kg_web graph with its cap of 50.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

from oracle import fastlog_oracle as O
from tests.conftest import GRAD_ATOL, GRAD_RTOL, exact_loop_grads, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
RTOL, ATOL = 1e-5, 1e-6


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV)


def _hubby():
    from minikg_dev_b200.synth import sample_graph
    kg = sample_graph(2500, 14, 60000, (("rel", ("zipf", 1.0)), ("head", (1.2, 3.0)), ("tail", (1.2, 3.0)),
                                        ("hubs", (0.02, 0.5))), seed=5, name="hubby")
    return kg.head, kg.rel, kg.tail, kg.num_entities, kg.num_relations


def _golden_g2():
    g = load_golden("g2")
    return g["head"], g["rel"], g["tail"], int(g["E"][0]), int(g["R"][0])


@pytest.fixture(params=["dense", "hash"])
def accum(request, monkeypatch):
    from minikg_dev_b200 import fastlog_kernel
    monkeypatch.setattr(fastlog_kernel, "ACCUM", request.param)
    return request.param


@pytest.mark.parametrize("graph", ["g2", "hubby"])
@pytest.mark.parametrize("cap,agg", [(O.UNCAPPED, 0), (3, 0), (40, 0), (O.UNCAPPED, 1), (3, 1)])
def test_hop_range_partition_union(graph, cap, agg, accum):
    from minikg_dev_b200.fastlog_kernel import HopRange
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.sharded import message_in_counts, plan_dst_ranges
    h, r, t, E, R = _golden_g2() if graph == "g2" else _hubby()
    g = DeviceGraph.from_triples(T(h), T(r), T(t), E, R)
    rng = np.random.default_rng(cap % 1000 + 7 * agg)
    B, L, n = 3, 2, 2 * R + 1
    w = rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32)
    keys = np.unique(rng.integers(0, B * L * E, 300))
    deg = np.bincount(h, minlength=E) + np.bincount(t, minlength=E)
    keys = np.unique(np.concatenate([keys, np.argsort(-deg)[:3] + E]))  # hubs in (b=0, l=1)
    fb, fl, fe = O.split3(keys, L, E)
    fv = rng.uniform(0.05, 1.0, keys.shape[0]).astype(np.float32)
    ew = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    ew[::4] = np.float32(0.5)
    bounds = plan_dst_ranges(message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E), 3)
    mk = torch.ones((), device=DEV)

    def run(lo, hi, seeds=None):
        sv = T(fv).requires_grad_(True)
        wt = T(w).requires_grad_(True)
        et = T(ew).requires_grad_(True)
        outs = HopRange.apply(T(fb), T(fl), T(fe), sv, wt, g, mk, et, B, L, False, cap, agg, True, 1.0, lo, hi)
        outs = [o.coalesce() for o in outs]
        res = [(O.keys3(*o.indices().cpu().numpy(), L, E), o.values().detach().cpu().numpy()) for o in outs]
        if seeds is not None and agg == 0:
            loss = 0
            for o, (k, _) in zip(outs, res):
                loss = loss + (o.values() * T(O.lookup(seeds[0], seeds[1], k))).sum()
            loss.backward()
            return res, (sv.grad.cpu().numpy(), wt.grad.cpu().numpy(), et.grad.cpu().numpy())
        return res, None

    full, _ = run(0, 0)
    all_keys = np.unique(np.concatenate([k for k, _ in full]))
    seeds = (all_keys, rng.standard_normal(all_keys.shape[0]).astype(np.float32))
    full, gfull = run(0, 0, seeds)
    parts, gsum = [], None
    for k in range(3):
        res, gr = run(bounds[k], bounds[k + 1], seeds)
        for kk, _ in res:
            assert ((kk % E >= bounds[k]) & (kk % E < bounds[k + 1])).all()
        parts.append(res)
        if gr is not None:
            gsum = gr if gsum is None else tuple(a + b for a, b in zip(gsum, gr))
    for j in range(3):
        k = np.concatenate([p[j][0] for p in parts])
        v = np.concatenate([p[j][1] for p in parts])
        o = np.argsort(k, kind="stable")
        np.testing.assert_array_equal(k[o], full[j][0])
        if agg == 1 and j < 2:
            np.testing.assert_array_equal(v[o], full[j][1])
        else:
            np.testing.assert_allclose(v[o], full[j][1], rtol=RTOL, atol=ATOL)
    if agg == 0:
        for a, b in zip(gsum, gfull):
            np.testing.assert_allclose(a, b, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("cap", [O.UNCAPPED, 3, 40])
def test_merged_hop_partition_union(cap, accum):
    """MergedHop (ori + inv + ind in one store) over a 3-way destination partition: the union is
    the full-range merged output, the gradients add up to the full-range ones, and the full
    output equals the oracle's concat-sum."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.sharded import message_in_counts, plan_dst_ranges
    from minikg_dev_b200.sparse_loop import MergedHop
    h, r, t, E, R = _hubby()
    g = DeviceGraph.from_triples(T(h), T(r), T(t), E, R)
    rng = np.random.default_rng(cap % 991)
    B, L, n = 3, 2, 2 * R + 1
    w = rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32)
    deg = np.bincount(h, minlength=E) + np.bincount(t, minlength=E)
    keys = np.unique(np.concatenate([rng.integers(0, B * L * E, 300), np.argsort(-deg)[:3] + E]))
    rng.shuffle(keys)  # the op takes frontier keys in any order
    fv = rng.uniform(0.05, 1.0, keys.shape[0]).astype(np.float32)
    ew = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    csr = O.build_csr_structure(h, t, r, E)
    fb, fl, fe = O.split3(keys, L, E)
    fwd = O.sparse3d_forward(fb, fl, fe, fv, w, csr, np.ones(h.shape[0], bool), ew, B, L, E, R, cap=cap,
                             is_score=True)
    want_k, want_v = O.sum_sparse3d_concat(fwd["ori"], fwd["inv"], fwd["ind"])
    seeds = rng.standard_normal(want_k.shape[0]).astype(np.float32)
    bounds = plan_dst_ranges(message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E), 3)

    def run(lo, hi):
        sv = T(fv).requires_grad_(True)
        wt = T(w).requires_grad_(True)
        et = T(ew).requires_grad_(True)
        k, v = MergedHop.apply(T(keys), sv, wt, et, g, None, True, 1.0, cap, lo, hi)
        kn = k.cpu().numpy()
        assert (np.diff(kn) > 0).all()
        (v * T(O.lookup(want_k, seeds, kn))).sum().backward()
        return kn, v.detach().cpu().numpy(), (sv.grad.cpu().numpy(), wt.grad.cpu().numpy(), et.grad.cpu().numpy())

    fk, fvv, fg = run(0, 0)
    np.testing.assert_array_equal(fk, want_k)
    np.testing.assert_allclose(fvv, want_v, rtol=RTOL, atol=ATOL)
    ks, vs, gsum = [], [], None
    for k in range(3):
        kk, vv, gr = run(bounds[k], bounds[k + 1])
        assert ((kk % E >= bounds[k]) & (kk % E < bounds[k + 1])).all()
        ks.append(kk)
        vs.append(vv)
        gsum = gr if gsum is None else tuple(a + b for a, b in zip(gsum, gr))
    np.testing.assert_array_equal(np.concatenate(ks)[np.argsort(np.concatenate(ks), kind="stable")], fk)
    for a, b in zip(gsum, fg):  # fp32 atomics in different orders over hub rows
        np.testing.assert_allclose(a, b, rtol=GRAD_RTOL, atol=GRAD_ATOL)


def test_hop_range_rejects_bad_range():
    from minikg_dev_b200.fastlog_kernel import HopRange
    from minikg_dev_b200.graph import DeviceGraph
    h, r, t, E, R = _golden_g2()
    g = DeviceGraph.from_triples(T(h), T(r), T(t), E, R)
    z = torch.zeros(1, dtype=torch.int64, device=DEV)
    w = torch.full((1, 1, 2 * R + 1), 0.1, device=DEV)
    with pytest.raises(RuntimeError, match="destination range"):
        HopRange.apply(z, z, z, torch.ones(1, device=DEV), w, g, torch.ones((), device=DEV), None, 1, 1, False,
                       O.UNCAPPED, 0, True, 1.0, 5, E + 1)


# ----------------------------------------------------------------------------- two GPUs
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, graph, case, out_q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from minikg_dev_b200 import sharded as S
        from minikg_dev_b200.graph import DeviceGraph
        h, r, t, E, R = graph
        heads, w, scores, cap, k = case
        tt = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
        g = DeviceGraph.from_triples(tt(h), tt(r), tt(t), E, R)
        bounds = S.plan_dst_ranges(S.message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E), world)
        spec = S.ShardSpec(rank, world, bounds)
        wt = tt(w).requires_grad_(True)
        ew = tt(scores).requires_grad_(True)
        hop = S.cuda_hop_fn(g, None, S.replicated(ew), cap, True, 1.0)
        keys, vals = S.sharded_proof_scores(spec, hop, tt(heads), wt, E)
        B = heads.shape[0]
        seed_all = torch.from_numpy(np.random.default_rng(99).standard_normal(B * E).astype(np.float32)).to(dev)
        (vals * seed_all[keys]).sum().backward()
        tails, sc, cnt = S.merge_topk(spec, keys, vals, B, E, k)
        torch.cuda.synchronize()
        out_q.put((rank, keys.cpu().numpy(), vals.detach().cpu().numpy(), wt.grad.cpu().numpy(),
                   ew.grad.cpu().numpy(), tails.cpu().numpy(), sc.cpu().numpy(), cnt.cpu().numpy()))
    finally:
        dist.destroy_process_group()


def test_sharded_loop_two_gpus_vs_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from minikg_dev_b200.synth import hop_inputs, sample_graph, scaled_workload
    wl = scaled_workload("kg_web", 0.02)
    kg = sample_graph(wl.E, wl.R, wl.T, wl.gen, seed=0, name=wl.name)
    E, R, B, L, K, cap, k = kg.num_entities, kg.num_relations, 8, wl.L, wl.hops, wl.capped_row, 20
    inp = hop_inputs(kg, B, L, K, seed=0)
    graph = (kg.head, kg.rel, kg.tail, E, R)
    case = (inp.heads, inp.rule_weights, inp.edge_scores, cap, k)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(rk, 2, port, graph, case, q)) for rk in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(2)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    csr = O.build_csr_structure(kg.head, kg.tail, kg.rel, E)
    mask = np.ones(kg.num_triples, bool)
    final, trace = O.proof_sum_forward(inp.heads, inp.rule_weights, csr, mask, inp.edge_scores, B, L, E, R, cap=cap)
    keys = np.concatenate([x[1] for x in res])
    vals = np.concatenate([x[2] for x in res])
    o = np.argsort(keys, kind="stable")
    keys, vals = keys[o], vals[o]
    np.testing.assert_array_equal(keys, final[0])
    np.testing.assert_allclose(vals, final[1], rtol=RTOL, atol=ATOL)
    seed_all = np.random.default_rng(99).standard_normal(B * E).astype(np.float32)
    gw, ge = exact_loop_grads(inp.heads, inp.rule_weights, csr, mask, inp.edge_scores, B, L, E, R, final[0],
                              seed_all[final[0]], num_facts=kg.num_triples, cap=cap)
    ot, osc, oc = O.decode_topk((keys, vals), B, E, k)
    for x in res:
        np.testing.assert_allclose(x[3], gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(x[4], ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_array_equal(x[5], ot)
        np.testing.assert_array_equal(x[6], osc)
        np.testing.assert_array_equal(x[7], oc)
