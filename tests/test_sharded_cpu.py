"""The destination-partitioned hop loop's host logic on CPU: world_size 2 (and 3) over gloo.

The per-rank hop here is the oracle's op restricted to the rank's destination range (an
autograd function around ``sparse3d_forward`` / ``sparse3d_backward``), so these tests check
the partition, the frontier all-gather and its gradient, the globally normalised columns,
the cross-rank prune and the top-k merge against the single-process oracle loop.  The CUDA
op in the same loop is checked on two GPUs in ``test_sharded_gpu.py``.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fastlog_oracle as O
from tests.conftest import GRAD_ATOL, GRAD_RTOL, exact_loop_grads, load_golden


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=0, B=5, L=3, K=3):
    g = load_golden("g2")
    h, r, t = g["head"], g["rel"], g["tail"]
    E, R = int(g["E"][0]), int(g["R"][0])
    rng = np.random.default_rng(seed)
    n = 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    heads[1] = heads[0]  # two queries from one head
    w = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    return h, r, t, E, R, heads, w, scores


class _OracleRangeHop(torch.autograd.Function):
    """The oracle hop (ori + inv + ind, concat-summed) with outputs restricted to destinations
    in [lo, hi): ``(keys, values)``, keys ascending."""

    @staticmethod
    def forward(ctx, keys, v, w_h, ew, csr, E, R, cap, lo, hi):
        B, L, _ = w_h.shape
        bn, ln, en = O.split3(keys.numpy(), L, E)
        vn = v.detach().numpy()
        wn, ewn = w_h.detach().numpy(), ew.detach().numpy()
        mask = np.ones(ewn.shape[0], bool)
        fwd = O.sparse3d_forward(bn, ln, en, vn, wn, csr, mask, ewn, B, L, E, R, cap=cap, agg_mode=0, is_score=True)
        parts = []
        for name in ("ori", "inv", "ind"):
            k, val = fwd[name]
            keep = ((k % E) >= lo) & ((k % E) < hi)
            parts.append((k[keep], val[keep]))
        mk, mv = O.sum_sparse3d_concat(*parts)
        ctx.fwd, ctx.args = fwd, (bn, ln, en, vn, wn, ewn, B, L, E, R)
        ctx.mk = mk
        out_k = torch.from_numpy(mk.astype(np.int64))
        ctx.mark_non_differentiable(out_k)
        return out_k, torch.from_numpy(mv.astype(np.float32))

    @staticmethod
    def backward(ctx, _gk, gv):
        bn, ln, en, vn, wn, ewn, B, L, E, R = ctx.args
        g = gv.numpy().astype(np.float32)
        grads = {name: (ctx.fwd[name][0], O.lookup(ctx.mk, g, ctx.fwd[name][0])) for name in ("ori", "inv", "ind")}
        gsp, gw, ge = O.sparse3d_backward(ctx.fwd, grads, bn, ln, en, vn, wn, B, L, E, R, agg_mode=0,
                                          edge_weight=ewn, is_score=True, want_edge_grad=True,
                                          num_facts=ewn.shape[0])
        return (None, torch.from_numpy(gsp), torch.from_numpy(gw), torch.from_numpy(ge),
                None, None, None, None, None, None)


def _worker(rank, world, port, cfg, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from minikg_dev_b200 import sharded as S
        h, r, t, E, R, heads, w, scores = _case(**cfg["case"])
        csr = O.build_csr_structure(h, t, r, E)
        bounds = S.plan_dst_ranges(S.message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E), world)
        spec = S.ShardSpec(rank, world, bounds)
        wt = torch.from_numpy(w).requires_grad_(True)
        ew = torch.from_numpy(scores).requires_grad_(True)
        ew_rep = S.replicated(ew)

        def hop(keys, v, w_h, lo, hi):
            return _OracleRangeHop.apply(keys, v, w_h, ew_rep, csr, E, R, cfg["cap"], lo, hi)

        keys, vals = S.sharded_proof_scores(spec, hop, torch.from_numpy(heads), wt, E, threshold=cfg["threshold"],
                                            topk_nodes=cfg["topk_nodes"])
        B = heads.shape[0]
        seed_all = np.random.default_rng(99).standard_normal(B * E).astype(np.float32)
        (vals * torch.from_numpy(seed_all)[keys]).sum().backward()
        tails, sc, cnt = S.merge_topk(spec, keys, vals, B, E, cfg["k"])
        out_q.put((rank, bounds, keys.numpy(), vals.detach().numpy(), wt.grad.numpy(), ew.grad.numpy(),
                   tails.numpy(), sc.numpy(), cnt.numpy()))
    finally:
        dist.destroy_process_group()


def _run(world, cfg):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(res, key=lambda x: x[0])


@pytest.mark.parametrize("world,cfg", [
    (2, dict(case=dict(seed=0), cap=O.UNCAPPED, threshold=0.0, topk_nodes=0, k=10)),
    (2, dict(case=dict(seed=1), cap=9, threshold=0.0, topk_nodes=0, k=25)),
    (3, dict(case=dict(seed=2), cap=O.UNCAPPED, threshold=1e-4, topk_nodes=0, k=10)),
    (2, dict(case=dict(seed=3), cap=O.UNCAPPED, threshold=0.0, topk_nodes=40, k=10)),
])
def test_sharded_loop_matches_single_process_oracle(world, cfg):
    h, r, t, E, R, heads, w, scores = _case(**cfg["case"])
    B, L = heads.shape[0], w.shape[2]
    csr = O.build_csr_structure(h, t, r, E)
    mask = np.ones(h.shape[0], bool)
    final, trace = O.proof_sum_forward(heads, w, csr, mask, scores, B, L, E, R, cap=cfg["cap"],
                                       topk_nodes=cfg["topk_nodes"], threshold=cfg["threshold"])
    res = _run(world, cfg)
    bounds = res[0][1]
    assert bounds[0] == 0 and bounds[-1] == E and all(a < b for a, b in zip(bounds, bounds[1:]))
    keys = np.concatenate([x[2] for x in res])
    vals = np.concatenate([x[3] for x in res])
    order = np.argsort(keys, kind="stable")  # ranks hold entity ranges; keys are b * E + e
    keys, vals = keys[order], vals[order]
    for rank, x in enumerate(res):  # every rank holds only its own entities
        assert ((x[2] % E >= bounds[rank]) & (x[2] % E < bounds[rank + 1])).all()
    np.testing.assert_array_equal(keys, final[0])
    np.testing.assert_allclose(vals, final[1], rtol=1e-5, atol=1e-6)
    seed_all = np.random.default_rng(99).standard_normal(B * E).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w, csr, mask, scores, B, L, E, R, final[0], seed_all[final[0]],
                              num_facts=h.shape[0], cap=cfg["cap"], topk_nodes=cfg["topk_nodes"],
                              threshold=cfg["threshold"])
    for x in res:  # the replicated inputs carry the full gradient on every rank
        np.testing.assert_allclose(x[4], gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(x[5], ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    # the merge is exact: compare with the oracle's decode of the same (gathered) raw scores
    ot, osc, oc = O.decode_topk((keys, vals), B, E, cfg["k"])
    for x in res:
        np.testing.assert_array_equal(x[6], ot)
        np.testing.assert_array_equal(x[7], osc)
        np.testing.assert_array_equal(x[8], oc)


def test_plan_dst_ranges_balances_messages():
    from minikg_dev_b200.sharded import message_in_counts, plan_dst_ranges
    h, r, t, E, R, *_ = _case()
    m = message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E)
    for world in (1, 2, 4, 8):
        b = plan_dst_ranges(m, world)
        assert b[0] == 0 and b[-1] == E and len(b) == world + 1
        assert all(x < y for x, y in zip(b, b[1:]))
        load = [int((m[b[k]:b[k + 1]] + 1).sum()) for k in range(world)]
        assert max(load) <= (int((m + 1).sum()) / world) + int(m.max()) + 1
    with pytest.raises(ValueError):
        plan_dst_ranges(torch.zeros(3, dtype=torch.int64), 4)


# ----------------------------------------------------------------------------- failures (host only)
def _fail_worker(rank, world, port, mode, out_q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    from minikg_dev_b200 import sharded as S
    h, r, t, E, R, heads, w, scores = _case(seed=4)
    csr = O.build_csr_structure(h, t, r, E)
    bounds = S.plan_dst_ranges(S.message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E), world)
    spec = S.ShardSpec(rank, world, bounds)
    if mode == "dead" and rank == 1:
        os._exit(0)  # the rank leaves between steps, with nothing in flight
    if mode == "size" and rank == 1:
        S._frontier_size = lambda keys: -5  # a corrupted size message
    ew = torch.from_numpy(scores)

    def hop(keys, v, w_h, lo, hi):
        return _OracleRangeHop.apply(keys, v, w_h, ew, csr, E, R, O.UNCAPPED, lo, hi)

    try:
        S.sharded_proof_scores(spec, hop, torch.from_numpy(heads), torch.from_numpy(w), E)
        out_q.put((rank, "no error"))
    except Exception as exc:  # noqa: BLE001 - the test inspects the error text
        out_q.put((rank, f"{type(exc).__name__}: {exc}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


@pytest.mark.parametrize("mode", ["dead", "size"])
def test_sharded_loop_reports_rank_failures(mode):
    """A rank that exits, or that sends an impossible frontier size, ends the other ranks'
    step with an error (process-group timeout 10 s, or the size check) instead of a hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    want = 1 if mode == "dead" else 2
    res = dict(q.get(timeout=120) for _ in range(want))
    for p in procs:
        p.join(timeout=60)
    assert res[0] != "no error"
    if mode == "size":
        assert "invalid frontier size" in res[0] and "invalid frontier size" in res[1]


# ----------------------------------------------------------------------------- slab frontier gather
def _gather_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from minikg_dev_b200.sharded import ShardSpec
        from minikg_dev_b200.slab_loop import _gather
        n = [3, 0, 5][rank]  # ragged, one rank empty
        keys = torch.arange(n, dtype=torch.int64) + 100 * rank
        vals = torch.tensor([-0.0, 1e-30, 3.5, float("inf"), 2.0 ** -126][:n], dtype=torch.float32) + 0.25 * rank
        k_all, v_all, off = _gather(keys, vals, ShardSpec(rank, world, [0, 10, 20, 30]))
        out_q.put((rank, k_all.numpy(), v_all.numpy().view(np.int32), off, vals.numpy().view(np.int32)))
    finally:
        dist.destroy_process_group()


def test_slab_frontier_gather_packs_keys_and_value_bits():
    """slab_loop._gather: one all-gather of [keys, fp32 bits] rows; every rank receives the
    ranks' lists concatenated in rank order, the values bit for bit, and its own offset."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(3)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_k = np.concatenate([np.arange([3, 0, 5][r]) + 100 * r for r in range(3)])
    want_v = np.concatenate([x[4] for x in res])
    for rank, k_all, v_bits, off, _ in res:
        np.testing.assert_array_equal(k_all, want_k)
        np.testing.assert_array_equal(v_bits, want_v)
        assert off == [0, 3, 3][rank]
