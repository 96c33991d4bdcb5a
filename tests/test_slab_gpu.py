"""Parity of the key-slab hop loop (``slab_loop.SlabHopLoop``, csrc/mkg_slab.cu) on the GPU.

The uncapped sum loop of proof.py:467-614 against the oracle: result keys and per-hop message
counts exact, values within rtol 1e-5 / atol 1e-6 of the fp32 oracle, rule-weight and
edge-score gradients within the same bar of the oracle's float64 run.  Also: the store's
row windows (a store too small for all rows), destination ranges whose union is the whole
hop, the store left zeroed after every use, and the loop over two GPUs with NCCL.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch

from oracle import fastlog_oracle as O
from tests.conftest import GRAD_ATOL, GRAD_RTOL, exact_loop_grads
from tests.test_gpu_parity import GRAPHS, T, csr_dev

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
DEV = torch.device("cuda", 0)


def _case(gname, B, L, K, seed, mask_frac=0.0):
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(seed)
    n = 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    mask = rng.random(h.shape[0]) >= mask_frac
    return h, r, t, E, R, heads, w_hops, scores, mask


def _engine(h, r, t, E, R, **kw):
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.slab_loop import SlabEngine
    csr = O.build_csr_structure(h, t, r, E)
    return csr, SlabEngine(DeviceGraph(csr_dev(csr), E, R), **kw)


def _store_is_zero(eng) -> bool:
    return eng.store is None or int(torch.count_nonzero(eng.store).item()) == 0


@pytest.mark.parametrize("gname,B,L,K,topk_nodes,thr,mask_frac", [
    ("hubby", 6, 3, 3, 0, 0.0, 0.0),
    ("g2", 6, 3, 3, 0, 0.0, 0.0),
    ("hubby", 40, 4, 2, 0, 0.0, 0.0),
    ("hubby", 6, 3, 3, 150, 0.0, 0.0),
    ("g2", 12, 3, 3, 0, 2e-3, 0.0),
    ("hubby", 8, 2, 3, 0, 0.0, 0.3),
])
def test_slab_loop_vs_oracle(gname, B, L, K, topk_nodes, thr, mask_frac):
    from minikg_dev_b200.slab_loop import slab_proof_scores
    h, r, t, E, R, heads, w_hops, scores, mask = _case(gname, B, L, K, B * 10 + K + topk_nodes, mask_frac)
    csr, eng = _engine(h, r, t, E, R)
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, topk_nodes=topk_nodes,
                                       threshold=thr)
    wt = T(w_hops).requires_grad_(True)
    sc = T(scores).requires_grad_(True)
    mk = T(mask.astype(np.float32)) if mask_frac > 0 else None
    out, msgs = slab_proof_scores(eng, T(heads), wt, sc, mk, True, 1.0, topk_nodes, thr)
    out = out.coalesce()
    idx = out.indices().cpu().numpy()
    got_k, got_v = idx[0] * E + idx[1], out.values().detach().cpu().numpy()
    if thr > 0:  # a value within rounding of the threshold may be kept by one summation order only
        common, ia, ib = np.intersect1d(got_k, final[0], return_indices=True)
        assert common.size >= final[0].size - 2 and common.size >= got_k.size - 2
        np.testing.assert_allclose(got_v[ia], final[1][ib], rtol=RTOL, atol=ATOL)
    else:
        np.testing.assert_array_equal(got_k, final[0])
        np.testing.assert_allclose(got_v, final[1], rtol=RTOL, atol=ATOL)
    assert msgs.cpu().tolist() == [O.count_messages(tr["state"], csr, w_hops[k], L, E, R)
                                   for k, tr in enumerate(trace)]
    seed = np.random.default_rng(7).standard_normal(got_k.shape[0]).astype(np.float32)
    (out.values() * T(seed)).sum().backward()
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, scores, B, L, E, R, got_k, seed, num_facts=h.shape[0],
                              topk_nodes=topk_nodes, threshold=thr)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    torch.cuda.synchronize()
    assert _store_is_zero(eng)


def test_slab_loop_row_windows_match_one_window():
    """A store of a few rows runs each hop window by window: same keys, values and gradients."""
    from minikg_dev_b200 import _native as N
    from minikg_dev_b200.slab_loop import slab_proof_scores
    h, r, t, E, R, heads, w_hops, scores, mask = _case("hubby", 9, 3, 3, 5)
    res = []
    for store_bytes in (None, int(N.load().mkg_slab_store_bytes(4 * E))):
        _, eng = _engine(h, r, t, E, R, store_bytes=store_bytes)
        wt = T(w_hops).requires_grad_(True)
        sc = T(scores).requires_grad_(True)
        out, msgs = slab_proof_scores(eng, T(heads), wt, sc)
        out = out.coalesce()
        (out.values() * torch.linspace(-1, 1, out.values().numel(), device=DEV)).sum().backward()
        res.append((out.indices(), out.values().detach(), msgs, wt.grad, sc.grad, eng.rows_per_window))
        assert _store_is_zero(eng)
    (i1, v1, m1, gw1, ge1, p1), (i2, v2, m2, gw2, ge2, p2) = res
    assert p1 == 27 and p2 == 4
    assert torch.equal(i1, i2) and torch.equal(m1, m2)
    np.testing.assert_allclose(v2.cpu().numpy(), v1.cpu().numpy(), rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gw2.cpu().numpy(), gw1.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(ge2.cpu().numpy(), ge1.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("tiles,store_rows", [(3, 0), (4, 4), (11, 0)])
def test_slab_loop_destination_tiles_match_one_tile(tiles, store_rows):
    """Destination tiles (each its own push list, walked tile by tile in one launch; 11 tiles
    take two launches, 8 + 3, the identity messages with the first), alone and with row
    windows: the same keys, values, message counts and gradients as one tile, and the
    oracle's."""
    from minikg_dev_b200 import _native as N
    from minikg_dev_b200.slab_loop import slab_proof_scores
    h, r, t, E, R, heads, w_hops, scores, mask = _case("hubby", 9, 3, 3, 41)
    res = []
    for kw in ({}, {"dst_tiles": tiles, **({"store_bytes": int(N.load().mkg_slab_store_bytes(store_rows * E))}
                                           if store_rows else {})}):
        csr, eng = _engine(h, r, t, E, R, **kw)
        wt = T(w_hops).requires_grad_(True)
        sc = T(scores).requires_grad_(True)
        out, msgs = slab_proof_scores(eng, T(heads), wt, sc)
        out = out.coalesce()
        (out.values() * torch.linspace(-1, 1, out.values().numel(), device=DEV)).sum().backward()
        res.append((out.indices(), out.values().detach(), msgs, wt.grad, sc.grad, len(eng.tiles)))
        assert _store_is_zero(eng)
    (i1, v1, m1, gw1, ge1, n1), (i2, v2, m2, gw2, ge2, n2) = res
    assert n1 == 1 and n2 == tiles
    assert torch.equal(i1, i2) and torch.equal(m1, m2)
    np.testing.assert_allclose(v2.cpu().numpy(), v1.cpu().numpy(), rtol=RTOL, atol=ATOL)
    final, _ = O.proof_sum_forward(heads, w_hops, csr, mask, scores, 9, 3, E, R)
    idx = i2.cpu().numpy()
    np.testing.assert_array_equal(idx[0] * E + idx[1], final[0])
    np.testing.assert_allclose(v2.cpu().numpy(), final[1], rtol=RTOL, atol=ATOL)
    seed = np.linspace(-1, 1, final[0].shape[0]).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, scores, 9, 3, E, R, final[0], seed, num_facts=h.shape[0])
    for gwx, gex in ((gw1, ge1), (gw2, ge2)):  # both against the float64 run (not one against the other)
        np.testing.assert_allclose(gwx.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(gex.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


def test_slab_hop_destination_ranges_add_up():
    """Engines holding only the push records of one destination range each: their hop outputs
    partition the whole-range output, and their row sums add up to its row sums."""
    from minikg_dev_b200.sharded import message_in_counts, plan_dst_ranges
    from minikg_dev_b200.slab_loop import expand_forward
    h, r, t, E, R, heads, w_hops, scores, mask = _case("hubby", 5, 3, 1, 11)
    csr, full = _engine(h, r, t, E, R)
    B, L = 5, 3
    full.set_edge_factor(None, T(scores), True, 1.0)
    rng = np.random.default_rng(3)
    keys = np.unique(rng.integers(0, B * L * E, 400))
    vals = rng.uniform(0.01, 1.0, keys.shape[0]).astype(np.float32)
    kf, vf, df, _ = expand_forward(full, T(keys), T(vals), T(w_hops[0]), B * L)
    # entity-major output: ascending entity, then row
    em = ((kf % E) * (B * L) + kf // E).cpu().numpy()
    assert (np.diff(em) > 0).all()
    o = torch.argsort(kf)
    kf, vf = kf[o], vf[o]
    bounds = plan_dst_ranges(message_in_counts(torch.from_numpy(h), torch.from_numpy(t), E), 3)
    ks, vs, ds = [], [], torch.zeros_like(df)
    from minikg_dev_b200.slab_loop import SlabEngine
    for k in range(3):
        eng = SlabEngine(full.g, bounds[k], bounds[k + 1])
        eng.set_edge_factor(None, T(scores), True, 1.0)
        kk, vv, dd, _ = expand_forward(eng, T(keys), T(vals), T(w_hops[0]), B * L)
        e = (kk % E).cpu().numpy()
        assert ((e >= bounds[k]) & (e < bounds[k + 1])).all()
        ks.append(kk)
        vs.append(vv)
        ds += dd
        assert _store_is_zero(eng)
    kc, vc = torch.cat(ks), torch.cat(vs)
    o = torch.argsort(kc)
    assert torch.equal(kc[o], kf)
    np.testing.assert_allclose(vc[o].cpu().numpy(), vf.cpu().numpy(), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(ds.cpu().numpy(), df.cpu().numpy(), rtol=1e-6, atol=1e-9)  # fp32 values summed in another order
    # the oracle's concat-sum of the same hop
    fb, fl, fe = O.split3(keys, L, E)
    fwd = O.sparse3d_forward(fb, fl, fe, vals, w_hops[0], csr, np.ones(h.shape[0], bool), scores, B, L, E, R,
                             is_score=True)
    want_k, want_v = O.sum_sparse3d_concat(fwd["ori"], fwd["inv"], fwd["ind"])
    nz = want_v != 0
    np.testing.assert_array_equal(kf.cpu().numpy(), want_k[nz])
    np.testing.assert_allclose(vf.cpu().numpy(), want_v[nz], rtol=RTOL, atol=ATOL)


def test_slab_bad_frontier_entity_is_reported():
    """A frontier key outside [B, L, E] is refused on the host; a negative key reaching the
    kernel is flagged, not followed, and the context stays usable; a key of a row outside the
    window belongs to another window's pass and is skipped without a flag."""
    import ctypes
    from minikg_dev_b200 import _native as N
    from minikg_dev_b200.slab_loop import _collect, expand_forward
    h, r, t, E, R, heads, w_hops, scores, mask = _case("g2", 2, 2, 1, 1)
    _, eng = _engine(h, r, t, E, R)
    keys = T(np.array([3, 2 * 2 * E + 5], np.int64))  # the second row is beyond B * L = 4
    with pytest.raises(RuntimeError, match="outside"):
        expand_forward(eng, keys, T(np.ones(2, np.float32)), T(w_hops[0]), 4)
    lib = N.load()
    eng.ensure_store(4)
    wf = T(w_hops[0]).reshape(4, -1).contiguous()

    def expand(win, k):
        v = T(np.ones(k.numel(), np.float32))
        ws = N.workspace(lib.mkg_slab_expand_workspace_bytes(k.numel()), DEV)
        _, _, ptr0, push0 = eng.tiles[0]
        N.check(lib.mkg_slab_expand(ptr0.data_ptr(), push0.data_ptr(), k.data_ptr(), v.data_ptr(), k.numel(),
                                    wf.data_ptr(), wf.shape[1], 1, 0, ctypes.byref(win), eng.store.data_ptr(), None,
                                    ws.data_ptr(), ws.numel(), N.error_word(DEV).data_ptr(), N.stream_handle(DEV)),
                "slab_expand")

    win = eng.window(0, 1)  # rows [0, 1)
    expand(win, T(np.array([3, -7], np.int64)))
    with pytest.raises(RuntimeError, match="outside"):
        N.raise_device_errors(DEV)
    _collect(eng, win)  # the accepted key's messages leave the store
    expand(win, T(np.array([3, E + 5], np.int64)))  # row 1: another window's entry
    N.raise_device_errors(DEV)
    ko, _ = _collect(eng, win)
    assert ko.numel() > 0 and bool(((ko // E) == 0).all())
    torch.cuda.synchronize()
    assert _store_is_zero(eng)


@pytest.mark.parametrize("gname,B,L,K,store_rows,tiles", [("hubby", 9, 3, 3, 0, 1), ("g2", 6, 3, 3, 0, 1),
                                                          ("hubby", 9, 3, 2, 4, 1), ("hubby", 9, 3, 3, 0, 3)])
def test_slab_decode_max_bit_exact(gname, B, L, K, store_rows, tiles):
    """The uncapped max-aggregation decode on the key-slab store (also window by window, and
    tile by tile): raw scores, tails and bounded scores bit-exact against the oracle."""
    from minikg_dev_b200 import _native as N
    from minikg_dev_b200.slab_loop import slab_decode_max
    h, r, t, E, R, heads, w_hops, scores, mask = _case(gname, B, L, K, 31 + B)
    kw = {"store_bytes": int(N.load().mkg_slab_store_bytes(store_rows * E))} if store_rows else {}
    kw["dst_tiles"] = tiles
    csr, eng = _engine(h, r, t, E, R, **kw)
    keys, raw, tails, sc, counts = slab_decode_max(eng, T(heads), T(w_hops), 20, T(scores))
    final, _ = O.proof_max_forward(heads, w_hops, csr, mask, scores, B, L, E, R)
    np.testing.assert_array_equal(keys.cpu().numpy(), final[0])
    np.testing.assert_array_equal(raw.cpu().numpy(), final[1])
    ot, osc, oc = O.decode_topk(final, B, E, 20)
    np.testing.assert_array_equal(tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(sc.cpu().numpy(), osc)
    np.testing.assert_array_equal(counts.cpu().numpy(), oc)
    torch.cuda.synchronize()
    assert _store_is_zero(eng)


# ----------------------------------------------------------------------------- two GPUs
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, case, out_q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from minikg_dev_b200.graph import DeviceGraph
        from minikg_dev_b200.sharded import ShardSpec, message_in_counts, plan_dst_ranges
        from minikg_dev_b200.slab_loop import SlabEngine, SlabHopLoop
        h, r, t, E, R, heads, w_hops, scores, topk_nodes = case
        tt = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
        g = DeviceGraph.from_triples(tt(h), tt(r), tt(t), E, R)
        bounds = plan_dst_ranges(message_in_counts(tt(h), tt(t), E), world)
        spec = ShardSpec(rank, world, bounds)
        eng = SlabEngine(g, spec.lo, spec.hi)
        wt = tt(w_hops).requires_grad_(True)
        sc = tt(scores).requires_grad_(True)
        keys, vals, msgs = SlabHopLoop.apply(wt, sc, tt(heads), eng, None, True, 1.0, topk_nodes, 0.0, spec)
        B = heads.shape[0]
        seed_all = torch.from_numpy(np.random.default_rng(99).standard_normal(B * E).astype(np.float32)).to(dev)
        (vals * seed_all[keys]).sum().backward()
        torch.cuda.synchronize()
        out_q.put((rank, keys.cpu().numpy(), vals.detach().cpu().numpy(), wt.grad.cpu().numpy(),
                   sc.grad.cpu().numpy(), msgs.cpu().numpy(), bounds))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("topk_nodes", [0, 150])
def test_slab_loop_two_gpus_vs_oracle(topk_nodes):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    h, r, t, E, R, heads, w_hops, scores, mask = _case("hubby", 7, 3, 3, 17)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    case = (h, r, t, E, R, heads, w_hops, scores, topk_nodes)
    procs = [ctx.Process(target=_rank_main, args=(rk, 2, port, case, q)) for rk in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(2)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    csr = O.build_csr_structure(h, t, r, E)
    B, L = heads.shape[0], w_hops.shape[2]
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, topk_nodes=topk_nodes)
    bounds = res[0][6]
    for rank, x in enumerate(res):
        e = x[1] % E
        assert ((e >= bounds[rank]) & (e < bounds[rank + 1])).all()
    keys = np.concatenate([x[1] for x in res])
    vals = np.concatenate([x[2] for x in res])
    o = np.argsort(keys, kind="stable")
    np.testing.assert_array_equal(keys[o], final[0])
    np.testing.assert_allclose(vals[o], final[1], rtol=RTOL, atol=ATOL)
    want_msgs = [O.count_messages(tr["state"], csr, w_hops[k], L, E, R) for k, tr in enumerate(trace)]
    seed_all = np.random.default_rng(99).standard_normal(B * E).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, scores, B, L, E, R, final[0], seed_all[final[0]],
                              num_facts=h.shape[0], topk_nodes=topk_nodes)
    for x in res:
        assert x[5].tolist() == want_msgs
        np.testing.assert_allclose(x[3], gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(x[4], ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


def _rule_sum_reference(keys, vals, E, L, take_max):
    """sum_sp_3d / max_sp_3d on an entity-major list, written out: each run of entries with
    one (e, b) folded in list order (fp32), the runs stably ordered by (b, e); each entry's
    output index."""
    e, b = keys % E, (keys // E) // L
    runs, owner = [], np.empty(keys.size, np.int64)
    i = 0
    while i < keys.size:
        acc, j = np.float32(vals[i]), i
        while j + 1 < keys.size and e[j + 1] == e[i] and b[j + 1] == b[i]:
            j += 1
            acc = np.maximum(acc, vals[j]) if take_max else np.float32(acc + vals[j])
        owner[i:j + 1] = len(runs)
        runs.append((b[i], e[i], acc))
        i = j + 1
    order = sorted(range(len(runs)), key=lambda r: (runs[r][0], runs[r][1]))
    rank = np.empty(len(runs), np.int64)
    rank[order] = np.arange(len(runs))
    out_k = np.array([runs[r][0] * E + runs[r][1] for r in order], np.int64)
    out_v = np.array([runs[r][2] for r in order], np.float32)
    return out_k, out_v, rank[owner] if keys.size else owner


def _rule_sum_gpu(keys, vals, E, L, B, take_max):
    from minikg_dev_b200 import _native as N
    lib = N.load()
    n = int(keys.size)
    k, v = T(keys), T(vals)
    ok = torch.empty(max(n, 1), dtype=torch.int64, device=DEV)
    ov = torch.empty(max(n, 1), dtype=torch.float32, device=DEV)
    pos = torch.empty(max(n, 1), dtype=torch.int64, device=DEV)
    cnt = torch.full((1,), -1, dtype=torch.int64, device=DEV)
    ws = N.workspace(lib.mkg_rule_sum_workspace_bytes(n), DEV)
    N.check(lib.mkg_rule_sum(N.ptr(k), N.ptr(v), n, E, L, B, int(take_max), ok.data_ptr(), ov.data_ptr(),
                             pos.data_ptr(), cnt.data_ptr(), N.ptr(ws), ws.numel(), N.error_word(DEV).data_ptr(),
                             N.stream_handle(DEV)), "rule_sum")
    N.raise_device_errors(DEV)
    U = int(cnt.item())
    return ok[:U].cpu().numpy(), ov[:U].cpu().numpy(), pos[:n].cpu().numpy()


@pytest.mark.parametrize("E,B,L,n,take_max", [
    (5000, 300, 4, 20000, False),   # counting placement: 10 blocks, runs across block and warp edges
    (5000, 300, 4, 20000, True),
    (900, 3, 2, 5000, False),       # many runs of one query in every warp item
    (4000, 1, 1, 3000, False),      # one rule, one query: every entry its own run
    (2000, 1500, 3, 12000, False),  # more queries than the counting placement takes: radix pipeline
    (2000, 1500, 3, 12000, True),
    (10, 4, 4, 0, False),           # empty
])
def test_rule_sum_entity_major(E, B, L, n, take_max):
    """mkg_rule_sum on entity-major lists (the slab emit's order) against the written-out fold:
    result keys, their positions and values bit-exact (fp32 sums in rule order; maxima)."""
    rng = np.random.default_rng(n + B)
    # about n entries: (e, b) pairs, each with a random non-empty subset of its L rules (runs of
    # 1 .. L entries), in entity-major order (ascending entity, then row)
    m = min(E * B, max(1, int(n / (0.7 * L + 0.3)))) if n else 0
    pairs = rng.choice(E * B, size=m, replace=False).astype(np.int64)
    take = rng.random((m, L)) < 0.7
    take[np.arange(m), rng.integers(0, L, m)] = True
    ii, ll = np.nonzero(take)
    keys = (pairs[ii] % B * L + ll) * E + pairs[ii] // B
    keys = keys[np.lexsort((keys // E, keys % E))].astype(np.int64)
    vals = rng.uniform(0.01, 1.0, keys.size).astype(np.float32)
    rk, rv, rpos = _rule_sum_reference(keys, vals, E, L, take_max)
    gk, gv, gpos = _rule_sum_gpu(keys, vals, E, L, B, take_max)
    np.testing.assert_array_equal(gk, rk)
    np.testing.assert_array_equal(gv.view(np.uint32), rv.view(np.uint32))
    np.testing.assert_array_equal(gpos, rpos)


def test_rule_sum_refuses_unordered_and_bad_keys():
    """An entry out of entity-major order, or outside [B, L, E], raises the device flag."""
    E, B, L = 50, 4, 2
    keys = np.array([0 * E + 3, 1 * E + 3, 0 * E + 7], np.int64)  # entity 3, 3, 7: ordered
    vals = np.ones(3, np.float32)
    _rule_sum_gpu(keys, vals, E, L, B, False)
    with pytest.raises(RuntimeError):
        _rule_sum_gpu(keys[[2, 0, 1]], vals, E, L, B, False)
    with pytest.raises(RuntimeError):
        _rule_sum_gpu(np.array([3, B * L * E + 1], np.int64), vals[:2], E, L, B, False)
