"""Parity of the CUDA path (through the C ABI) against the oracle and the golden vectors.

Bar: integer / index / argmax / bucketing / decode results bit-exact; fp32 sums and
gradients within rtol 1e-5, atol 1e-6.  Hop-loop gradients are held to that bar against the
oracle run in float64 arithmetic (``exact_loop_grads``): the reference's own fp32 result is a
rounding of that value and already lies up to a few times the bar away from it after three
hops of sums (measured in test_oracle_golden.py).
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from oracle import fastlog_oracle as O
from tests.conftest import GRAD_ATOL, GRAD_RTOL, exact_loop_grads, load_golden, softmax_backward

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 1e-6
UNC = O.UNCAPPED
DEV = torch.device("cuda", 0)


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from minikg_dev_b200 import _native
    _native.load()


@pytest.fixture(params=["dense", "hash"])
def accum(request, monkeypatch):
    """The per-hop op's message store: key slab or hash tables."""
    from minikg_dev_b200 import fastlog_kernel
    monkeypatch.setattr(fastlog_kernel, "ACCUM", request.param)
    return request.param


def T(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.to(DEV, dtype=dtype) if dtype is not None else t.to(DEV)


def coo_np(sp, L, E):
    sp = sp.coalesce()
    idx = sp.indices().cpu().numpy()
    return O.keys3(idx[0], idx[1], idx[2], L, E), sp.values().detach().cpu().numpy()


def csr_dev(csr_np):
    return tuple(T(a) for a in csr_np)


def graphs():
    from minikg_dev_b200.synth import sample_graph
    out = {}
    for name in ("g1", "g2"):
        g = load_golden(name)
        out[name] = (g["head"], g["rel"], g["tail"], int(g["E"][0]), int(g["R"][0]))
    kg = sample_graph(2500, 14, 60000, (("rel", ("zipf", 1.0)), ("head", (1.2, 3.0)), ("tail", (1.2, 3.0)),
                                        ("hubs", (0.02, 0.5))), seed=5, name="hubby")
    out["hubby"] = (kg.head, kg.rel, kg.tail, kg.num_entities, kg.num_relations)
    return out


GRAPHS = graphs()


# ----------------------------------------------------------------------------- CSR build
@pytest.mark.parametrize("name", list(GRAPHS))
def test_csr_build_bit_exact(name):
    from minikg_dev_b200.graph import build_csr_structure
    h, r, t, E, R = GRAPHS[name]
    mine = build_csr_structure(T(h), T(t), T(r), E, R)
    want = O.build_csr_structure(h, t, r, E)
    for k in range(16):
        np.testing.assert_array_equal(mine[k].cpu().numpy().astype(np.int64), want[k].astype(np.int64),
                                      err_msg=f"csr{k}")


def test_ind2ptr():
    from minikg_dev_b200.graph import ind2ptr
    rng = np.random.default_rng(3)
    idx = np.sort(rng.integers(0, 50, 400))
    np.testing.assert_array_equal(ind2ptr(T(idx), 60).cpu().numpy(), O.ind2ptr(idx, 60))
    np.testing.assert_array_equal(ind2ptr(T(np.empty(0, np.int64)), 5).cpu().numpy(), np.zeros(6))


# ----------------------------------------------------------------------------- per-hop op
def run_op(csr_np, E, R, fb, fl, fe, fv, w, mask, ew, cap, agg, is_score, wot_i=False, scale=1.0,
           seeds=None):
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    B, L, n = w.shape
    sv = T(fv).requires_grad_(True)
    wt = T(w).requires_grad_(True)
    ewt = T(ew).requires_grad_(True) if ew is not None else None
    mk = T(mask.astype(np.float32)) if mask is not None else torch.ones((), device=DEV)
    o, i, d = FastLogFunctionSparse3DTopK.apply(T(fb), T(fl), T(fe), sv, wt, *csr_dev(csr_np), mk, ewt, B, L, E,
                                                R, wot_i, int(cap), int(agg), bool(is_score), float(scale))
    res = {"ori": coo_np(o, L, E), "inv": coo_np(i, L, E), "ind": coo_np(d, L, E)}
    if seeds is not None:
        loss = 0
        for name, t in (("ori", o), ("inv", i), ("ind", d)):
            t = t.coalesce()
            loss = loss + (t.values() * T(seeds[name])).sum()
        loss.backward()
        res["grad_sp"] = sv.grad.cpu().numpy()
        res["grad_w"] = wt.grad.cpu().numpy()
        res["grad_edge"] = ewt.grad.cpu().numpy() if ewt is not None else None
    return res


OP_CASES = [("sum_unc", UNC, 0, True), ("sum_cap", 7, 0, True), ("max_unc", UNC, 1, True),
            ("max_cap", 7, 1, True), ("sum_logit", UNC, 0, False), ("sum_cap0", 0, 0, True)]


@pytest.mark.parametrize("gname", ["g1", "g2"])
@pytest.mark.parametrize("tag,cap,agg,is_score", OP_CASES)
def test_hop_op_vs_golden(gname, tag, cap, agg, is_score, accum):
    """The op against the reference's own outputs on the golden inputs."""
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    w = g["op_w"]
    B, L, _ = w.shape
    csr = tuple(g[f"csr{k}"] for k in range(16))
    seeds = {n: g[f"{tag}_seed_{n}"] for n in ("ori", "inv", "ind")}
    res = run_op(csr, E, R, g["op_b"], g["op_l"], g["op_e"], g["op_v"], w, np.ones(g["head"].shape[0], bool),
                 g[tag + "_ew"], cap, agg, is_score, seeds=seeds)
    for name in ("ori", "inv", "ind"):
        idx = g[f"{tag}_{name}_idx"]
        want_k = O.keys3(idx[0], idx[1], idx[2], L, E)
        np.testing.assert_array_equal(res[name][0], want_k, err_msg=name)
        if agg == 1 and name != "ind":
            np.testing.assert_array_equal(res[name][1], g[f"{tag}_{name}_val"], err_msg=name)
        else:
            tol = 1e-6 if is_score else 2e-6  # sigmoid path: CUDA double-rounded sigmoid vs torch's
            np.testing.assert_allclose(res[name][1], g[f"{tag}_{name}_val"], rtol=tol, atol=1e-7, err_msg=name)
    np.testing.assert_allclose(res["grad_sp"], g[tag + "_grad_sp"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(res["grad_w"], g[tag + "_grad_w"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(res["grad_edge"], g[tag + "_grad_edge"], rtol=RTOL, atol=ATOL)


def _frontier(rng, B, L, E, per_row, dup_values=True):
    rows = []
    for b in range(B):
        for l in range(L):
            for e in rng.choice(E, size=min(per_row, E), replace=False):
                rows.append((b, l, int(e)))
    a = np.array(sorted(rows), np.int64).reshape(-1, 3)
    v = rng.uniform(0.05, 1.0, a.shape[0]).astype(np.float32)
    if dup_values:
        v[::5] = np.float32(0.25)
    return a[:, 0].copy(), a[:, 1].copy(), a[:, 2].copy(), v


@pytest.mark.parametrize("gname", ["hubby", "g2"])
@pytest.mark.parametrize("cap,agg", [(UNC, 0), (UNC, 1), (3, 0), (3, 1), (40, 0), (1, 1), (0, 0)])
@pytest.mark.parametrize("variant", ["plain", "zero_mask", "wot_i", "logit"])
def test_hop_op_vs_oracle(gname, cap, agg, variant, accum):
    """Synthetic inputs with hubs (block-per-entry path), masked facts (explicit zero
    outputs), the wot_i flag and the sigmoid edge path."""
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(zlib.crc32(f"{gname}/{cap}/{agg}/{variant}".encode()))
    csr = O.build_csr_structure(h, t, r, E)
    B, L = 3, 2
    n = 2 * R + 1
    w = O.F32(1.0) * (rng.dirichlet(np.ones(n), size=(B, L))).astype(np.float32)
    w[0, 0, :] = w[0, 0, 0]  # equal weights: many exact message ties
    fb, fl, fe, fv = _frontier(rng, B, L, E, per_row=40)
    # make sure the biggest hubs are in the frontier
    deg = np.bincount(h, minlength=E) + np.bincount(t, minlength=E)
    hubs = np.argsort(-deg)[:3]
    extra = np.array([(0, 1, int(x)) for x in hubs], np.int64)
    allk = np.unique(np.concatenate([O.keys3(fb, fl, fe, L, E), O.keys3(extra[:, 0], extra[:, 1], extra[:, 2], L, E)]))
    fb, fl, fe = O.split3(allk, L, E)
    fv = rng.uniform(0.05, 1.0, allk.shape[0]).astype(np.float32)
    T_ = h.shape[0]
    mask = np.ones(T_, bool)
    if variant == "zero_mask":
        mask[rng.random(T_) < 0.3] = False
    is_score = variant != "logit"
    ew = rng.uniform(0.05, 1.0, T_).astype(np.float32) if is_score else rng.standard_normal(T_).astype(np.float32)
    if is_score:
        ew[::4] = np.float32(0.5)
    wot_i = variant == "wot_i"
    scale = 0.7 if variant == "logit" else 1.0
    fwd = O.sparse3d_forward(fb, fl, fe, fv, w, csr, mask, ew, B, L, E, R, wot_i=wot_i, cap=cap, agg_mode=agg,
                             is_score=is_score, scale=scale)
    seeds = {name: rng.standard_normal(fwd[name][0].shape[0]).astype(np.float32) for name in ("ori", "inv", "ind")}
    res = run_op(csr, E, R, fb, fl, fe, fv, w, mask, ew, cap, agg, is_score, wot_i=wot_i, scale=scale, seeds=seeds)
    for name in ("ori", "inv", "ind"):
        np.testing.assert_array_equal(res[name][0], fwd[name][0], err_msg=name)
        if agg == 1 and name != "ind" and is_score:
            np.testing.assert_array_equal(res[name][1], fwd[name][1], err_msg=name)
        else:
            np.testing.assert_allclose(res[name][1], fwd[name][1], rtol=RTOL, atol=ATOL, err_msg=name)
    grads = {name: (fwd[name][0], seeds[name]) for name in ("ori", "inv", "ind")}
    gsp, gw, ge = O.sparse3d_backward(fwd, grads, fb, fl, fe, fv, w, B, L, E, R, wot_i=wot_i, agg_mode=agg,
                                      edge_weight=ew, is_score=is_score, scale=scale, want_edge_grad=True,
                                      num_facts=T_)
    np.testing.assert_allclose(res["grad_sp"], gsp, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(res["grad_w"], gw, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(res["grad_edge"], ge, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("mode", ["dense", "hash"])
def test_hop_op_argmax_facts_bit_exact(mode):
    """The argmax message per key (smallest fact id among equal maxima) through the C ABI."""
    import ctypes
    from minikg_dev_b200 import _native as N
    from minikg_dev_b200.graph import DeviceGraph
    h, r, t, E, R = GRAPHS["hubby"]
    csr = O.build_csr_structure(h, t, r, E)
    rng = np.random.default_rng(9)
    B, L, n = 2, 2, 2 * R + 1
    w = np.full((B, L, n), 0.05, np.float32)  # all channels equal: ties everywhere
    fb, fl, fe, fv = _frontier(rng, B, L, E, per_row=30)
    fv[:] = np.float32(0.5)
    ew = np.full(h.shape[0], 0.5, np.float32)
    fwd = O.sparse3d_forward(fb, fl, fe, fv, w, csr, np.ones(h.shape[0], bool), ew, B, L, E, R, agg_mode=1,
                             is_score=True)
    g = DeviceGraph(csr_dev(csr), E, R)
    keep = [T(fb), T(fl), T(fe), T(fv)]
    fr = N.Frontier(*(x.data_ptr() for x in keep), fb.shape[0])
    wt = T(w)
    f = N.edge_factor(None, T(ew), True, 1.0, keep)
    p = N.HopParams(B, L, E, R, n, 0, 1, UNC)
    lib = N.load()
    if mode == "hash":
        mc = torch.empty(2, dtype=torch.int64, device=DEV)
        N.check(lib.mkg_hop_count_messages(ctypes.byref(g.struct), ctypes.byref(fr), ctypes.byref(p), mc.data_ptr(),
                                           N.error_word(DEV).data_ptr(), None), "count")
        p.msg_bound, p.accum = int(mc.max()), 2
        assert int(mc.sum()) == O.count_messages((O.keys3(fb, fl, fe, L, E), fv), csr, w, L, E, R)
    ws = N.workspace(lib.mkg_hop_forward_workspace_bytes(ctypes.byref(p), fb.shape[0]), DEV)
    counts = torch.zeros(3, dtype=torch.int64, device=DEV)
    N.check(lib.mkg_hop_forward(ctypes.byref(g.struct), ctypes.byref(fr), wt.data_ptr(), ctypes.byref(f),
                                ctypes.byref(p), ws.data_ptr(), ws.numel(), counts.data_ptr(),
                                N.error_word(DEV).data_ptr(), None), "hop_forward")
    sizes = counts.tolist()
    for which, name in ((0, "ori"), (1, "inv")):
        U = sizes[which]
        idx = torch.empty((3, U), dtype=torch.int64, device=DEV)
        val = torch.empty(U, dtype=torch.float32, device=DEV)
        arg = torch.empty(U, dtype=torch.int64, device=DEV)
        N.check(lib.mkg_hop_emit(ctypes.byref(p), fb.shape[0], ws.data_ptr(), ws.numel(), which, U, idx.data_ptr(),
                                 val.data_ptr(), arg.data_ptr(), None), "hop_emit")
        raw = fwd["raw_" + name]
        np.testing.assert_array_equal(arg.cpu().numpy(), raw["edge"][fwd[name + "_arg"]])
        np.testing.assert_array_equal(val.cpu().numpy(), fwd[name][1])


def test_hop_op_empty_frontier(accum):
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    h, r, t, E, R = GRAPHS["g1"]
    csr = csr_dev(O.build_csr_structure(h, t, r, E))
    e = torch.empty(0, dtype=torch.int64, device=DEV)
    w = torch.full((2, 2, 2 * R + 1), 0.1, device=DEV)
    o, i, d = FastLogFunctionSparse3DTopK.apply(e, e, e, torch.empty(0, device=DEV), w, *csr,
                                                torch.ones(h.shape[0], device=DEV), None, 2, 2, E, R, False, UNC, 0)
    assert o._nnz() == 0 and i._nnz() == 0 and d._nnz() == 0


def test_hash_table_overflow_is_reported_not_faulted():
    """A message bound below the real count fills the table: flagged, messages dropped, no fault."""
    import ctypes
    from minikg_dev_b200 import _native as N
    from minikg_dev_b200.graph import DeviceGraph
    h, r, t, E, R = GRAPHS["hubby"]
    csr = O.build_csr_structure(h, t, r, E)
    g = DeviceGraph(csr_dev(csr), E, R)
    rng = np.random.default_rng(2)
    B, L, n = 4, 4, 2 * R + 1
    fb, fl, fe, fv = _frontier(rng, B, L, E, per_row=40)
    keep = [T(fb), T(fl), T(fe), T(fv)]
    fr = N.Frontier(*(x.data_ptr() for x in keep), fb.shape[0])
    w = T(np.full((B, L, n), 0.05, np.float32))
    f = N.edge_factor(None, None, True, 1.0, keep)
    p = N.HopParams(B, L, E, R, n, 0, 0, UNC, 0, 0, 1, 2)  # bound 1: a 1024-slot table per direction
    lib = N.load()
    ws = N.workspace(lib.mkg_hop_forward_workspace_bytes(ctypes.byref(p), fb.shape[0]), DEV)
    counts = torch.zeros(3, dtype=torch.int64, device=DEV)
    N.check(lib.mkg_hop_forward(ctypes.byref(g.struct), ctypes.byref(fr), w.data_ptr(), ctypes.byref(f),
                                ctypes.byref(p), ws.data_ptr(), ws.numel(), counts.data_ptr(),
                                N.error_word(DEV).data_ptr(), None), "hop_forward")
    with pytest.raises(RuntimeError, match="ran out of slots"):
        N.raise_device_errors(DEV)
    assert counts.tolist()[0] <= 1024
    assert torch.ones(4, device=DEV).sum().item() == 4.0


def test_bad_index_is_reported_not_faulted():
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    h, r, t, E, R = GRAPHS["g1"]
    csr = csr_dev(O.build_csr_structure(h, t, r, E))
    b = torch.tensor([0, 0], device=DEV)
    l = torch.tensor([0, 0], device=DEV)
    ent = torch.tensor([1, E + 5], device=DEV)  # second entity is out of range
    w = torch.full((1, 1, 2 * R + 1), 0.1, device=DEV)
    with pytest.raises(RuntimeError, match="outside"):
        FastLogFunctionSparse3DTopK.apply(b, l, ent, torch.ones(2, device=DEV), w, *csr, torch.ones((), device=DEV),
                                          None, 1, 1, E, R, False, UNC, 0)
    torch.cuda.synchronize()  # the context is still usable
    assert torch.ones(4, device=DEV).sum().item() == 4.0


# ----------------------------------------------------------------------------- fused loop
def _w_hops_from_logits(logits):
    lg = torch.from_numpy(logits)
    return np.stack([torch.softmax(lg[:, t], dim=-1).numpy() for t in range(lg.shape[1])])


@pytest.mark.parametrize("gname", ["g1", "g2"])
def test_fused_loop_vs_golden(gname):
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import proof_scores
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    heads, logits, scores = g["pr_heads"], g["pr_logits"], g["pr_scores"]
    B, K, L, n = logits.shape
    dg = DeviceGraph(csr_dev(tuple(g[f"csr{k}"] for k in range(16))), E, R)
    lg = T(logits).requires_grad_(True)
    w_hops = torch.stack([torch.softmax(lg[:, t], dim=-1) for t in range(K)])
    sc = T(scores).requires_grad_(True)
    out, msgs = proof_scores(dg, T(heads), w_hops, sc, mask=torch.ones(g["head"].shape[0], device=DEV))
    idx = g["pr_unc_final_idx"]
    dense = np.zeros((B, E), np.float32)
    dense[idx[0], idx[1]] = g["pr_unc_final_val"]
    got = out.detach().cpu().numpy()
    np.testing.assert_array_equal(got != 0, dense != 0)
    np.testing.assert_allclose(got, dense, rtol=RTOL, atol=ATOL)
    seed = np.zeros((B, E), np.float32)
    seed[idx[0], idx[1]] = g["pr_unc_seed"]
    (out * T(seed)).sum().backward()
    # gradients: against the float64 run of the oracle on the golden inputs (the oracle's fp32
    # run is pinned to the golden gradients in test_oracle_golden.py)
    w_np = w_hops.detach().cpu().numpy()
    csr = tuple(g[f"csr{k}"] for k in range(16))
    gw, ge = exact_loop_grads(heads, w_np, csr, np.ones(g["head"].shape[0], bool), scores, B, L, E, R,
                              idx[0] * E + idx[1], g["pr_unc_seed"], num_facts=g["head"].shape[0])
    gl = softmax_backward(w_np, gw).transpose(1, 0, 2, 3)  # [K, B, L, n] -> [B, K, L, n]
    np.testing.assert_allclose(lg.grad.cpu().numpy(), gl, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("gname,B,L,K", [(g, *s) for g in ("hubby", "g2") for s in ((5, 3, 3), (40, 4, 2))] +
                         # 32 queries x 40 rules: a seed block's column segment spans 1,280 columns
                         # (> 256 float4s), the backward seed's multi-pass path with global S sums
                         [("g2", 32, 40, 2)])
def test_fused_loop_vs_oracle(gname, B, L, K):
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import proof_scores
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(B * 100 + K)
    csr = O.build_csr_structure(h, t, r, E)
    n = 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    mask = np.ones(h.shape[0], bool)
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R)
    dg = DeviceGraph(csr_dev(csr), E, R)
    wt = T(w_hops).requires_grad_(True)
    sc = T(scores).requires_grad_(True)
    out, msgs = proof_scores(dg, T(heads), wt, sc, mask=None)
    want = np.zeros((B, E), np.float32)
    b, e = final[0] // E, final[0] % E
    want[b, e] = final[1]
    got = out.detach().cpu().numpy()
    np.testing.assert_array_equal(got != 0, want != 0)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    exp_msgs = [O.count_messages(tr["state"], csr, w_hops[k], L, E, R) for k, tr in enumerate(trace)]
    assert msgs.cpu().tolist() == exp_msgs
    seed = rng.standard_normal(final[0].shape[0]).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, scores, B, L, E, R, final[0], seed, num_facts=h.shape[0])
    gd = np.zeros((B, E), np.float32)
    gd[b, e] = seed
    (out * T(gd)).sum().backward()
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("gname", ["hubby", "g2"])
@pytest.mark.parametrize("cap,topk_nodes", [(UNC, 0), (9, 0), (40, 150), (3, 0), (0, 0)])
def test_sparse_loop_vs_oracle(gname, cap, topk_nodes, accum):
    """The fused sparse hop loop (merged op outputs, written-out backward) against the oracle."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.sparse_loop import sparse_proof_scores
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(cap % 997 + topk_nodes)
    csr = O.build_csr_structure(h, t, r, E)
    B, L, K, n = 6, 3, 3, 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    mask = np.ones(h.shape[0], bool)
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, cap=cap, topk_nodes=topk_nodes)
    dg = DeviceGraph(csr_dev(csr), E, R)
    wt = T(w_hops).requires_grad_(True)
    sc = T(scores).requires_grad_(True)
    out, msgs = sparse_proof_scores(dg, T(heads), wt, sc, None, True, 1.0, cap, topk_nodes)
    out = out.coalesce()
    idx = out.indices().cpu().numpy()
    np.testing.assert_array_equal(idx[0] * E + idx[1], final[0])
    np.testing.assert_allclose(out.values().detach().cpu().numpy(), final[1], rtol=RTOL, atol=ATOL)
    assert msgs.cpu().tolist() == [O.count_messages(tr["state"], csr, w_hops[k], L, E, R, cap=cap)
                                   for k, tr in enumerate(trace)]
    seed = rng.standard_normal(final[0].shape[0]).astype(np.float32)
    (out.values() * T(seed)).sum().backward()
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, scores, B, L, E, R, final[0], seed, num_facts=h.shape[0],
                              cap=cap, topk_nodes=topk_nodes)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("gname", ["hubby", "g2"])
@pytest.mark.parametrize("cap", [0, 1, 3, 9, 40])
def test_fused_capped_loop_vs_oracle(gname, cap):
    """The fused dense loop with the edge cap (per-hop take tables of the capped rows)."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import proof_scores
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(cap + 7)
    csr = O.build_csr_structure(h, t, r, E)
    B, L, K, n = 12, 3, 3, 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    w_hops[:, 1, 0, :] = np.float32(1.0 / n)  # every group of a row in one bucket: ties decided by group order
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    mask = np.ones(h.shape[0], bool)
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, cap=cap)
    dg = DeviceGraph(csr_dev(csr), E, R)
    wt = T(w_hops).requires_grad_(True)
    sc = T(scores).requires_grad_(True)
    out, msgs = proof_scores(dg, T(heads), wt, sc, mask=None, topk_edges=cap)
    want = np.zeros((B, E), np.float32)
    b, e = final[0] // E, final[0] % E
    want[b, e] = final[1]
    got = out.detach().cpu().numpy()
    np.testing.assert_array_equal(got != 0, want != 0)
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    assert msgs.cpu().tolist() == [O.count_messages(tr["state"], csr, w_hops[k], L, E, R, cap=cap)
                                   for k, tr in enumerate(trace)]
    seed = rng.standard_normal(final[0].shape[0]).astype(np.float32)
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, scores, B, L, E, R, final[0], seed, num_facts=h.shape[0],
                              cap=cap)
    gd = np.zeros((B, E), np.float32)
    gd[b, e] = seed
    (out * T(gd)).sum().backward()
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


@pytest.mark.parametrize("gname", ["hubby", "g2"])
def test_cap_index_sizes(gname):
    """Capped rows (out-degree above the cap, per direction) and their relation groups."""
    from minikg_dev_b200.graph import DeviceGraph
    h, r, t, E, R = GRAPHS[gname]
    csr = O.build_csr_structure(h, t, r, E)
    dg = DeviceGraph(csr_dev(csr), E, R)
    for cap in (0, 3, 40, 255):
        slots = groups = 0
        capdeg = np.zeros(E, np.int64)
        for rp, gp in ((csr[0], csr[8]), (csr[4], csr[12])):
            deg = np.diff(rp.astype(np.int64))
            ng = np.diff(gp.astype(np.int64))
            slots += int((deg > cap).sum())
            groups += int(ng[deg > cap].sum())
            capdeg += np.minimum(deg, cap)
        ix = dg.cap_index(cap)
        assert (ix.num_slots, ix.num_groups) == (slots, groups)
        np.testing.assert_array_equal(dg._cap[cap][1]["capped_degree"][:E].cpu().numpy(), capdeg)


@pytest.mark.parametrize("gname", ["hubby", "g2"])
@pytest.mark.parametrize("cap", [1, 9, 40])
def test_fused_capped_max_decode_vs_oracle_bit_exact(gname, cap):
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(31 + cap)
    csr = O.build_csr_structure(h, t, r, E)
    B, L, K, n = 16, 3, 3, 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    w_hops[:, 0, 0, :] = np.float32(1.0 / n)
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    scores[::3] = np.float32(0.5)
    final, _ = O.proof_max_forward(heads, w_hops, csr, np.ones(h.shape[0], bool), scores, B, L, E, R, cap=cap)
    dg = DeviceGraph(csr_dev(csr), E, R)
    res = decode_max(dg, T(heads), T(w_hops), 100, T(scores), topk_edges=cap)
    want = np.zeros((B, E), np.float32)
    want[final[0] // E, final[0] % E] = final[1]
    np.testing.assert_array_equal(res.raw.cpu().numpy(), want)
    ot, osc, oc = O.decode_topk(final, B, E, 100)
    np.testing.assert_array_equal(res.tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(res.scores.cpu().numpy(), osc)
    np.testing.assert_array_equal(res.counts.cpu().numpy(), oc)


@pytest.mark.parametrize("gname", ["g1", "g2"])
def test_fused_capped_max_decode_vs_golden(gname):
    """The fused capped decode on the reference's own CSR (its in-group order decides which
    edges a capped group takes) against the reference's capped decode (cap 9)."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    heads, logits, scores = g["pr_heads"], g["pr_logits"], g["pr_scores"]
    B, K, L, n = logits.shape
    dg = DeviceGraph(csr_dev(tuple(g[f"csr{k}"] for k in range(16))), E, R)
    k = g["dec_cap_tails"].shape[1]
    res = decode_max(dg, T(heads), T(_w_hops_from_logits(logits)), k, T(scores), topk_edges=9)
    idx = g["dec_cap_final_idx"]
    want = np.zeros((B, E), np.float32)
    want[idx[0], idx[1]] = g["dec_cap_final_val"]
    np.testing.assert_array_equal(res.raw.cpu().numpy(), want)
    np.testing.assert_array_equal(res.tails.cpu().numpy(), g["dec_cap_tails"])
    np.testing.assert_allclose(res.scores.cpu().numpy(), g["dec_cap_scores"], rtol=0, atol=6e-8)


@pytest.mark.parametrize("gname", ["g1", "g2"])
def test_max_decode_vs_golden_bit_exact(gname):
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    heads, logits, scores = g["pr_heads"], g["pr_logits"], g["pr_scores"]
    B, K, L, n = logits.shape
    w_hops = _w_hops_from_logits(logits)
    dg = DeviceGraph(csr_dev(tuple(g[f"csr{k}"] for k in range(16))), E, R)
    k = g["dec_unc_tails"].shape[1]
    res = decode_max(dg, T(heads), T(w_hops), k, T(scores), mask=None)
    idx = g["dec_unc_final_idx"]
    want = np.zeros((B, E), np.float32)
    want[idx[0], idx[1]] = g["dec_unc_final_val"]
    np.testing.assert_array_equal(res.raw.cpu().numpy(), want)
    # oracle decode of the same raw scores: bit-exact; golden: tails exact, scores within one exp ulp
    ot, osc, oc = O.decode_topk((idx[0] * E + idx[1], g["dec_unc_final_val"]), B, E, k)
    np.testing.assert_array_equal(res.tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(res.scores.cpu().numpy(), osc)
    np.testing.assert_array_equal(res.counts.cpu().numpy(), oc)
    np.testing.assert_array_equal(res.tails.cpu().numpy(), g["dec_unc_tails"])
    np.testing.assert_allclose(res.scores.cpu().numpy(), g["dec_unc_scores"], rtol=0, atol=6e-8)


@pytest.mark.parametrize("gname", ["hubby", "g2"])
def test_max_decode_vs_oracle_bit_exact(gname):
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max
    h, r, t, E, R = GRAPHS[gname]
    rng = np.random.default_rng(17)
    csr = O.build_csr_structure(h, t, r, E)
    B, L, K, n = 24, 3, 3, 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    w_hops[:, 0, 0, :] = np.float32(1.0 / n)  # a tie-heavy query
    scores = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
    scores[::3] = np.float32(0.5)
    final, _ = O.proof_max_forward(heads, w_hops, csr, np.ones(h.shape[0], bool), scores, B, L, E, R)
    dg = DeviceGraph(csr_dev(csr), E, R)
    res = decode_max(dg, T(heads), T(w_hops), 100, T(scores))
    want = np.zeros((B, E), np.float32)
    want[final[0] // E, final[0] % E] = final[1]
    np.testing.assert_array_equal(res.raw.cpu().numpy(), want)
    ot, osc, oc = O.decode_topk(final, B, E, 100)
    np.testing.assert_array_equal(res.tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(res.scores.cpu().numpy(), osc)
    np.testing.assert_array_equal(res.counts.cpu().numpy(), oc)


@pytest.mark.parametrize("gname", ["g1", "g2"])
@pytest.mark.parametrize("tag,cap", [("dec_unc", UNC), ("dec_cap", 9)])
def test_max_decode_sparse_vs_golden_bit_exact(gname, tag, cap, accum):
    """The hop-by-hop max decode (any cap) against the reference's own outputs, on the
    reference's CSR (its order inside a capped group decides which edges are taken)."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max_sparse
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    heads, logits, scores = g["pr_heads"], g["pr_logits"], g["pr_scores"]
    B, K, L, n = logits.shape
    dg = DeviceGraph(csr_dev(tuple(g[f"csr{k}"] for k in range(16))), E, R)
    k = g[tag + "_tails"].shape[1]
    final, tails, sc, counts = decode_max_sparse(dg, T(heads), T(_w_hops_from_logits(logits)), k, T(scores),
                                                 mask=torch.ones(g["head"].shape[0], device=DEV), cap=cap)
    idx = final.indices().cpu().numpy()
    np.testing.assert_array_equal(idx, g[tag + "_final_idx"])
    np.testing.assert_array_equal(final.values().cpu().numpy(), g[tag + "_final_val"])
    keys = idx[0] * E + idx[1]
    ot, osc, oc = O.decode_topk((keys, final.values().cpu().numpy()), B, E, k)
    np.testing.assert_array_equal(tails.cpu().numpy(), ot)
    np.testing.assert_array_equal(sc.cpu().numpy(), osc)
    np.testing.assert_array_equal(counts.cpu().numpy(), oc)
    np.testing.assert_array_equal(tails.cpu().numpy(), g[tag + "_tails"])
    np.testing.assert_allclose(sc.cpu().numpy(), g[tag + "_scores"], rtol=0, atol=6e-8)


def test_decode_topk_ties_and_short_rows():
    from minikg_dev_b200.proof import decode_topk
    rng = np.random.default_rng(4)
    B, E = 6, 3000
    raw = np.zeros((B, E), np.float32)
    for b in range(B):
        m = [5, 150, 2999, 0, 1000, 7][b]
        cols = rng.choice(E, m, replace=False)
        raw[b, cols] = rng.choice(np.array([0.5, 0.25, 1.5, 3.0, 1e-9], np.float32), m)
    for k in (1, 10, 100, 1024):
        tails, scores, counts = decode_topk(T(raw), k)
        keys = np.nonzero(raw.reshape(-1))[0]
        ot, osc, oc = O.decode_topk((keys, raw.reshape(-1)[keys]), B, E, k)
        np.testing.assert_array_equal(tails.cpu().numpy(), ot)
        np.testing.assert_array_equal(scores.cpu().numpy(), osc)
        np.testing.assert_array_equal(counts.cpu().numpy(), oc)


def test_sparse_topk_ties_zeros_and_short_rows():
    """mkg_sparse_topk (k <= 1024) and the sort path (k > 1024) against the oracle's decode on a
    sparse state: explicit zeros and negative values are candidates with score 0, tied scores
    order by tail, empty rows and rows shorter than k, keys of rows past B ignored."""
    from minikg_dev_b200.proof import sparse_topk
    rng = np.random.default_rng(6)
    B, E = 7, 5000
    keys, vals = [], []
    for b in range(B + 1):  # row B lies outside the batch
        m = [5, 150, 4999, 0, 1300, 7, 2048, 40][b]
        cols = np.sort(rng.choice(E, m, replace=False))
        keys.append(b * E + cols)
        vals.append(rng.choice(np.array([0.5, 0.25, 1.5, 3.0, 1e-9, 0.0, -2.0], np.float32), m))
    keys, vals = np.concatenate(keys).astype(np.int64), np.concatenate(vals)
    inside = keys < B * E
    for k in (1, 10, 100, 1024, 1500):
        tails, scores, counts = sparse_topk(T(keys), T(vals), B, E, k)
        ot, osc, oc = O.decode_topk((keys[inside], vals[inside]), B, E, k)
        np.testing.assert_array_equal(tails.cpu().numpy(), ot)
        np.testing.assert_array_equal(scores.cpu().numpy(), osc)
        np.testing.assert_array_equal(counts.cpu().numpy(), oc)
    tails, scores, counts = sparse_topk(T(keys[:0]), T(vals[:0]), B, E, 5)
    assert counts.sum().item() == 0 and (tails == -1).all().item()


# ----------------------------------------------------------------------------- drop-in
@pytest.mark.parametrize("gname", ["g1", "g2"])
@pytest.mark.parametrize("tag,cap,topk_nodes", [("pr_unc", UNC, 0), ("pr_cap", 9, 0), ("pr_prune", UNC, 40)])
def test_kernel_sparse_scores_drop_in(gname, tag, cap, topk_nodes, accum):
    """The reference's hop driver signature, with a duck-typed model / graph / args."""
    from types import SimpleNamespace
    from minikg_dev_b200.proof import kernel_sparse_scores
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    heads, logits, scores = g["pr_heads"], g["pr_logits"], g["pr_scores"]
    B, K, L, n = logits.shape
    lg = T(logits).requires_grad_(True)
    wt = T(scores).requires_grad_(True)
    model = SimpleNamespace(rules=L, entity_count=E, relation_count=R, step=K, tau_1=1.0, weight=wt,
                            dropout=torch.nn.Identity(), build_rule_logits=lambda rels: lg)
    head_t, rel_t, tail_t = T(g["head"]), T(g["rel"]), T(g["tail"])
    mask = torch.ones(head_t.shape[0], dtype=torch.bool, device=DEV)
    graph = SimpleNamespace(e2triple=(head_t, None, mask), triple2e=(None, tail_t, mask), r2triple=(rel_t, None, mask),
                            mask=mask, mask_float=mask.float())
    args = SimpleNamespace(kernel_topk_edges=cap, kernel_topk_nodes=topk_nodes)
    out = kernel_sparse_scores(model, T(heads), T(np.zeros(B, np.int64)), graph, args, is_training=True)
    out = out.coalesce()
    idx = out.indices().cpu().numpy()
    gi = g[tag + "_final_idx"]
    if cap >= UNC:  # the build's CSR order inside a (row, rel) group may differ only when a cap cuts a group
        np.testing.assert_array_equal(idx, gi)
        np.testing.assert_allclose(out.values().detach().cpu().numpy(), g[tag + "_final_val"], rtol=RTOL, atol=ATOL)
        (out.values() * T(g[tag + "_seed"])).sum().backward()
        w_np = _w_hops_from_logits(logits)
        csr = tuple(g[f"csr{k}"] for k in range(16))
        gw, ge = exact_loop_grads(heads, w_np, csr, np.ones(g["head"].shape[0], bool), scores, B, L, E, R,
                                  idx[0] * E + idx[1], g[tag + "_seed"], num_facts=g["head"].shape[0],
                                  topk_nodes=topk_nodes)
        gl = softmax_backward(w_np, gw).transpose(1, 0, 2, 3)
        np.testing.assert_allclose(lg.grad.cpu().numpy(), gl, rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(wt.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    else:
        # capped: compare against the oracle on the build's own (stable) CSR
        csr = O.build_csr_structure(g["head"], g["tail"], g["rel"], E)
        w_hops = _w_hops_from_logits(logits)
        final, _ = O.proof_sum_forward(heads, w_hops, csr, np.ones(g["head"].shape[0], bool), scores, B, L, E, R,
                                       cap=cap, topk_nodes=topk_nodes)
        np.testing.assert_array_equal(idx[0] * E + idx[1], final[0])
        np.testing.assert_allclose(out.values().detach().cpu().numpy(), final[1], rtol=RTOL, atol=ATOL)


# ----------------------------------------------------------------------------- degenerate graphs
def test_isolated_entities_and_factless_graph():
    """Entities without edges send nothing but their identity message, through the op, the
    fused loop, the sparse loop and the decode; on a graph with no facts at all the op emits the
    identity output only (the reference's CSR build cannot take an empty fact list either)."""
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max, proof_scores
    from minikg_dev_b200.sparse_loop import sparse_proof_scores
    E, R = 50, 3
    B, L, n = 2, 2, 2 * R + 1
    w = np.full((B, L, n), 1.0 / n, np.float32)
    fb = np.array([0, 0, 1], np.int64)
    fl = np.array([0, 1, 1], np.int64)
    fe = np.array([10, 0, 49], np.int64)  # 10 and 49 have no edges
    fv = np.array([0.5, 1.0, 0.25], np.float32)
    for hh, rr, tt in ((np.array([0, 1, 2]), np.array([0, 1, 2]), np.array([1, 2, 3])),
                       (np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros(0, np.int64))):
        csr = O.build_csr_structure(hh, tt, rr, E)
        dg = DeviceGraph(csr_dev(csr), E, R)
        scores = np.full(hh.size, 0.5, np.float32)
        ew = T(scores) if hh.size else None
        o, i, d = FastLogFunctionSparse3DTopK.apply(T(fb), T(fl), T(fe), T(fv), T(w), *dg.csr,
                                                    torch.ones((), device=DEV), ew, B, L, E, R, False, UNC, 0,
                                                    True, 1.0)
        fwd = O.sparse3d_forward(fb, fl, fe, fv, w, csr, np.ones(hh.size, bool), scores if hh.size else None,
                                 B, L, E, R, is_score=True)
        for name, tns in (("ori", o), ("inv", i), ("ind", d)):
            k3, v3 = coo_np(tns, L, E)
            np.testing.assert_array_equal(k3, fwd[name][0])
            np.testing.assert_allclose(v3, fwd[name][1], rtol=RTOL, atol=ATOL)
        if not hh.size:
            assert o._nnz() == 0 and i._nnz() == 0 and d._nnz() == 3
            continue
        heads = T(np.array([10, 0], np.int64))
        w_hops = T(np.stack([w, w]))
        out, msgs = proof_scores(dg, heads, w_hops, ew)
        sp, _ = sparse_proof_scores(dg, heads, w_hops, ew, cap=2)
        final, trace = O.proof_sum_forward(np.array([10, 0]), np.stack([w, w]), csr, np.ones(3, bool), scores,
                                           B, L, E, R)
        want = np.zeros((B, E), np.float32)
        want[final[0] // E, final[0] % E] = final[1]
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(sp.to_dense().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
        assert out[0, 10].item() > 0  # the isolated head keeps its identity mass
        res = decode_max(dg, heads, w_hops, 5, ew)
        assert int(res.tails[0, 0]) == 10 and int(res.counts[0]) == 1


def test_device_graph_from_npy(tmp_path):
    """The .npy fact-file loader streams in chunks and builds the same CSR as the oracle."""
    from minikg_dev_b200.graph import DeviceGraph
    h, r, t, E, R = GRAPHS["g2"]
    facts = np.stack([h, r, t], 1).astype(np.int64)
    path = tmp_path / "all_id.npy"
    np.save(path, facts)
    g = DeviceGraph.from_npy(path, DEV, chunk=1000)
    assert g.num_entities == int(max(h.max(), t.max())) + 1 and g.num_relations == int(r.max()) + 1
    want = O.build_csr_structure(h, t, r, g.num_entities)
    for k, (got, exp) in enumerate(zip(g.csr, want)):
        np.testing.assert_array_equal(got.cpu().numpy(), exp, err_msg=f"csr[{k}]")


@pytest.mark.parametrize("variant", ["mask", "logit", "threshold"])
@pytest.mark.parametrize("engine", ["fused", "fused_capped", "sparse"])
def test_loops_masked_facts_and_sigmoid_path(variant, engine):
    """Both hop loops (the fused one uncapped and with cap 9) with facts masked off (their
    messages are explicit zeros, dropped by the normalisation), with the sigmoid edge-score
    path, or with a state threshold, against the oracle, fwd and bwd."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import proof_scores
    from minikg_dev_b200.sparse_loop import sparse_proof_scores
    h, r, t, E, R = GRAPHS["hubby"]
    rng = np.random.default_rng(31)
    csr = O.build_csr_structure(h, t, r, E)
    B, L, K, n = 6, 3, 3, 2 * R + 1
    heads = rng.integers(0, E, B).astype(np.int64)
    w_hops = np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])
    mask = np.ones(h.shape[0], bool)
    thr = 0.0
    if variant == "logit":
        ew = rng.standard_normal(h.shape[0]).astype(np.float32)
        is_score, scale = False, 0.7
    else:
        if variant == "mask":
            mask[rng.random(h.shape[0]) < 0.3] = False
        else:
            thr = 2e-3
        ew = rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)
        is_score, scale = True, 1.0
    if variant == "threshold" and engine == "sparse":
        pytest.skip("the sparse loop's threshold is covered by the workload tests")
    cap = UNC if engine == "fused" else 9
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, ew, B, L, E, R, cap=cap, is_score=is_score,
                                       scale=scale, threshold=thr)
    dg = DeviceGraph(csr_dev(csr), E, R)
    wt = T(w_hops).requires_grad_(True)
    sc = T(ew).requires_grad_(True)
    mk = T(mask.astype(np.float32))
    if engine != "sparse":
        out, _ = proof_scores(dg, T(heads), wt, sc, mask=mk, is_score=is_score, scale=scale, threshold=thr,
                              topk_edges=cap)
        got = out.detach().cpu().numpy()
        want = np.zeros((B, E), np.float32)
        want[final[0] // E, final[0] % E] = final[1]
        np.testing.assert_array_equal(got != 0, want != 0)
        np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
        seed = rng.standard_normal(final[0].shape[0]).astype(np.float32)
        gd = np.zeros((B, E), np.float32)
        gd[final[0] // E, final[0] % E] = seed
        (out * T(gd)).sum().backward()
    else:
        out, _ = sparse_proof_scores(dg, T(heads), wt, sc, mk, is_score, scale, cap, 0)
        idx = out.indices().cpu().numpy()
        np.testing.assert_array_equal(idx[0] * E + idx[1], final[0])
        np.testing.assert_allclose(out.values().detach().cpu().numpy(), final[1], rtol=RTOL, atol=ATOL)
        seed = rng.standard_normal(final[0].shape[0]).astype(np.float32)
        (out.values() * T(seed)).sum().backward()
    gw, ge = exact_loop_grads(heads, w_hops, csr, mask, ew, B, L, E, R, final[0], seed, num_facts=h.shape[0],
                              cap=cap, is_score=is_score, scale=scale, threshold=thr)
    np.testing.assert_allclose(wt.grad.cpu().numpy(), gw, rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(sc.grad.cpu().numpy(), ge, rtol=GRAD_RTOL, atol=GRAD_ATOL)


# ----------------------------------------------------------------------------- tracing, determinism
def test_reference_trace_flags(monkeypatch, capsys):
    """FASTLOG_STAGE_TIMING / FASTLOG_SPARSE_DEBUG_COUNTS print the reference's lines, with the
    raw message counts the reference's fill kernel would produce."""
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    monkeypatch.setenv("FASTLOG_STAGE_TIMING", "1")
    monkeypatch.setenv("FASTLOG_SPARSE_DEBUG_COUNTS", "1")
    h, r, t, E, R = GRAPHS["hubby"]
    csr = O.build_csr_structure(h, t, r, E)
    rng = np.random.default_rng(12)
    B, L, n = 3, 2, 2 * R + 1
    w = rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32)
    fb, fl, fe, fv = _frontier(rng, B, L, E, per_row=20)
    FastLogFunctionSparse3DTopK.apply(T(fb), T(fl), T(fe), T(fv), T(w), *csr_dev(csr), torch.ones((), device=DEV),
                                      None, B, L, E, R, False, 7, 0)
    out = capsys.readouterr().out
    for stage in ("prepare_inputs", "cuda_forward", "save_ctx"):
        assert f"StageTiming fastlog_kernel stage:sparse3d_topk.{stage} seconds:" in out
    fwd = O.sparse3d_forward(fb, fl, fe, fv, w, csr, np.ones(h.shape[0], bool), None, B, L, E, R, cap=7)
    line = [x for x in out.splitlines() if x.startswith("Sparse3DTopKCounts")][0]
    assert line == (f"Sparse3DTopKCounts nnz={fb.shape[0]} ori_total={fwd['raw_ori']['edge'].shape[0]} "
                    f"inv_total={fwd['raw_inv']['edge'].shape[0]} ind_total={fb.shape[0]}")


def test_argmax_paths_are_deterministic():
    """Max values, argmax facts and the decode are identical across repeated runs; the sum
    paths' keys are identical (their fp32 values may differ in the last bits)."""
    from minikg_dev_b200.fastlog_bridge import FastLogFunctionSparse3DTopK
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import decode_max, proof_scores
    h, r, t, E, R = GRAPHS["hubby"]
    csr = O.build_csr_structure(h, t, r, E)
    dg = DeviceGraph(csr_dev(csr), E, R)
    rng = np.random.default_rng(13)
    B, L, K, n = 8, 3, 3, 2 * R + 1
    heads = T(rng.integers(0, E, B).astype(np.int64))
    w_hops = T(np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)]))
    sc = T(rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32))
    runs = [decode_max(dg, heads, w_hops, 50, sc) for _ in range(3)]
    for res in runs[1:]:
        assert torch.equal(res.raw, runs[0].raw) and torch.equal(res.tails, runs[0].tails)
        assert torch.equal(res.scores, runs[0].scores)
    fb, fl, fe, fv = _frontier(rng, 2, L, E, per_row=30)
    outs = [FastLogFunctionSparse3DTopK.apply(T(fb), T(fl), T(fe), T(fv), w_hops[0][:2], *dg.csr,
                                              torch.ones((), device=DEV), sc, 2, L, E, R, False, 5, 1, True, 1.0)
            for _ in range(3)]
    for o in outs[1:]:
        for a, b in zip(o, outs[0]):
            assert torch.equal(a.coalesce().indices(), b.coalesce().indices())
            assert torch.equal(a.coalesce().values(), b.coalesce().values())
    s1, _ = proof_scores(dg, heads, w_hops, sc)
    s2, _ = proof_scores(dg, heads, w_hops, sc)
    assert torch.equal(s1 != 0, s2 != 0)


def test_fused_step_graph_replay_matches_eager():
    """ProofRunner.capture: a replayed step equals the eager step, and new inputs written into
    the captured buffers are picked up by the replay."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import ProofRunner
    h, r, t, E, R = GRAPHS["g2"]
    csr = O.build_csr_structure(h, t, r, E)
    dg = DeviceGraph(csr_dev(csr), E, R)
    rng = np.random.default_rng(21)
    B, L, K, n = 6, 3, 3, 2 * R + 1
    runner = ProofRunner(dg, B, L, K)
    heads = T(rng.integers(0, E, B).astype(np.int64))
    w_hops = T(np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)]))
    sc = T(rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32))
    G = T(rng.standard_normal((B, E)).astype(np.float32))
    out = torch.empty((B, E), device=DEV)
    msgs = torch.zeros(K, dtype=torch.int64, device=DEV)
    gw = torch.empty((K, B, L, n), device=DEV)
    ge = torch.empty(h.shape[0], device=DEV)
    graph = runner.capture(heads, w_hops, out, msgs, G, sc, gw, ge)
    for trial in range(2):
        if trial == 1:  # new inputs in place
            heads.copy_(T(rng.integers(0, E, B).astype(np.int64)))
            w_hops.copy_(T(np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)])))
        graph.replay()
        torch.cuda.synchronize()
        got = (out.clone(), gw.clone(), ge.clone())
        dg.set_edge_factor(None, sc, True, 1.0)
        o2, _ = runner.forward(heads, w_hops)
        gw2, ge2 = runner.backward(G, None, sc, True, 1.0, True)
        np.testing.assert_allclose(got[0].cpu().numpy(), o2.cpu().numpy(), rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(got[1].cpu().numpy(), gw2.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(got[2].cpu().numpy(), ge2.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)


def test_fused_step_graph_host_copies():
    """ProofRunner.capture with host_inputs / host_outputs: inputs written into the pinned host
    tensors reach the replay, results land in the pinned host outputs and equal the eager step;
    a host tensor that is not pinned is refused."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import ProofRunner
    h, r, t, E, R = GRAPHS["g2"]
    csr = O.build_csr_structure(h, t, r, E)
    dg = DeviceGraph(csr_dev(csr), E, R)
    rng = np.random.default_rng(22)
    B, L, K, n = 5, 2, 3, 2 * R + 1
    runner = ProofRunner(dg, B, L, K)

    def draw():
        return (torch.from_numpy(rng.integers(0, E, B).astype(np.int64)),
                torch.from_numpy(np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32)
                                           for _ in range(K)])),
                torch.from_numpy(rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32)))

    hh, wh, sh = (x.pin_memory() for x in draw())
    heads, w_hops, sc = hh.to(DEV), wh.to(DEV), sh.to(DEV)
    G = T(rng.standard_normal((B, E)).astype(np.float32))
    out = torch.empty((B, E), device=DEV)
    msgs = torch.zeros(K, dtype=torch.int64, device=DEV)
    gw = torch.empty((K, B, L, n), device=DEV)
    ge = torch.empty(h.shape[0], device=DEV)
    mh = torch.empty(K, dtype=torch.int64).pin_memory()
    gwh = torch.empty((K, B, L, n)).pin_memory()
    geh = torch.empty(h.shape[0]).pin_memory()
    with pytest.raises(ValueError, match="pinned"):
        runner.capture(heads, w_hops, out, msgs, G, sc, gw, ge, host_inputs=[(heads, torch.zeros(B, dtype=torch.int64))])
    graph = runner.capture(heads, w_hops, out, msgs, G, sc, gw, ge,
                           host_inputs=[(heads, hh), (w_hops, wh), (sc, sh)],
                           host_outputs=[(mh, msgs), (gwh, gw), (geh, ge)])
    for trial in range(2):
        if trial == 1:  # new inputs in the host tensors only
            for dst, src in zip((hh, wh, sh), draw()):
                dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        got = (mh.clone(), gwh.clone(), geh.clone())
        heads2, w2, sc2 = hh.to(DEV), wh.to(DEV), sh.to(DEV)
        dg.set_edge_factor(None, sc2, True, 1.0)
        _, m2 = runner.forward(heads2, w2)
        gw2, ge2 = runner.backward(G, None, sc2, True, 1.0, True)
        assert torch.equal(got[0], m2.cpu())
        np.testing.assert_allclose(got[1].numpy(), gw2.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)
        np.testing.assert_allclose(got[2].numpy(), ge2.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)


def test_fused_step_after_denser_step_matches_fresh_runner():
    """The normalisation skips the state chunks that hold no value and leaves them as an earlier
    step wrote them: a sparse step run after a dense one on the same runner equals the same step
    on a fresh runner.  The three 128-column chunks get different heads, so rows whose chunk is
    set next to an empty sibling chunk (both read by the 8-column forward lanes) occur."""
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import ProofRunner
    h, r, t, E, R = GRAPHS["hubby"]
    csr = O.build_csr_structure(h, t, r, E)
    dg = DeviceGraph(csr_dev(csr), E, R)
    rng = np.random.default_rng(23)
    B, L, K, n = 100, 3, 3, 2 * R + 1

    def weights():
        return T(np.stack([rng.dirichlet(np.ones(n), size=(B, L)).astype(np.float32) for _ in range(K)]))

    sc = T(rng.uniform(0.05, 1.0, h.shape[0]).astype(np.float32))
    G = T(rng.standard_normal((B, E)).astype(np.float32))
    used = ProofRunner(dg, B, L, K)
    dg.set_edge_factor(None, sc, True, 1.0)
    used.forward(T(rng.integers(0, E, B).astype(np.int64)), weights())
    used.backward(G, None, sc, True, 1.0, True)
    heads = T(np.repeat(rng.choice(E, 3, replace=False), [43, 43, 14]).astype(np.int64))
    w_hops = weights()
    res = []
    for runner in (used, ProofRunner(dg, B, L, K)):
        dg.set_edge_factor(None, sc, True, 1.0)
        o, m = runner.forward(heads, w_hops)
        gw, ge = runner.backward(G, None, sc, True, 1.0, True)
        res.append((o.clone(), m.clone(), gw.clone(), ge.clone()))
    (o1, m1, gw1, ge1), (o2, m2, gw2, ge2) = res
    assert torch.equal(m1, m2)
    np.testing.assert_allclose(o1.cpu().numpy(), o2.cpu().numpy(), rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(gw1.cpu().numpy(), gw2.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)
    np.testing.assert_allclose(ge1.cpu().numpy(), ge2.cpu().numpy(), rtol=GRAD_RTOL, atol=GRAD_ATOL)


# ----------------------------------------------------------------------------- decode candidates
@pytest.mark.parametrize("gname", ["g1", "g2"])
@pytest.mark.parametrize("cap", [UNC, 9])
def test_iter_decode_candidate_batches(gname, cap):
    """decode_core.py:394-420 on the device: per microbatch every candidate of every row, bounded
    and ordered (score desc, tail asc); against the oracle's sum loop + bound per row."""
    from types import SimpleNamespace
    from minikg_dev_b200.decode import iter_decode_candidate_batches, ordered_candidates
    g = load_golden(gname)
    E, R = int(g["E"][0]), int(g["R"][0])
    heads, logits, scores = g["pr_heads"], g["pr_logits"], g["pr_scores"]
    B, K, L, n = logits.shape
    lg = T(logits)
    model = SimpleNamespace(rules=L, entity_count=E, relation_count=R, step=K, tau_1=1.0, weight=T(scores),
                            dropout=torch.nn.Identity(), build_rule_logits=lambda rels: lg[rels])
    head_t, rel_t, tail_t = T(g["head"]), T(g["rel"]), T(g["tail"])
    mask = torch.ones(head_t.shape[0], dtype=torch.bool, device=DEV)
    graph = SimpleNamespace(e2triple=(head_t, None, mask), triple2e=(None, tail_t, mask), r2triple=(rel_t, None, mask),
                            mask=mask, mask_float=mask.float())
    args = SimpleNamespace(kernel_topk_edges=cap, kernel_topk_nodes=0, decode_proof_microbatch_size=4)
    rows = {}
    for a, b, cand in iter_decode_candidate_batches(model, T(heads), torch.arange(B, device=DEV), graph, args):
        assert (a, b) in [(0, 4), (4, B)]
        rows.update({a + r: v for r, v in cand.items()})
    csr = O.build_csr_structure(g["head"], g["tail"], g["rel"], E)
    final, _ = O.proof_sum_forward(heads, _w_hops_from_logits(logits), csr, np.ones(g["head"].shape[0], bool), scores,
                                   B, L, E, R, cap=cap)
    ot, osc, oc = O.decode_topk(final, B, E, E)
    for r in range(B):
        tails, sc = rows.get(r, (np.zeros(0, np.int64), np.zeros(0, np.float32)))
        assert tails.size == oc[r]
        want = dict(zip(ot[r, : oc[r]].tolist(), osc[r, : oc[r]].tolist()))
        assert sorted(tails.tolist()) == sorted(want)
        np.testing.assert_allclose(sc, [want[t] for t in tails.tolist()], rtol=1e-5, atol=1e-7)
        # decode order on the device's own scores: score descending, then tail ascending
        assert all((sc[i] > sc[i + 1]) or (sc[i] == sc[i + 1] and tails[i] < tails[i + 1]) for i in range(sc.size - 1))
    # a capped candidate list is the prefix of the full one
    raw = torch.zeros((B, E), device=DEV)
    raw[torch.from_numpy(final[0] // E), torch.from_numpy(final[0] % E)] = T(final[1])
    full_t, full_s, full_c = ordered_candidates(raw, 0)
    top_t, top_s, top_c = ordered_candidates(raw, 5)
    np.testing.assert_array_equal(top_c.cpu().numpy(), np.minimum(full_c.cpu().numpy(), 5))
    np.testing.assert_array_equal(top_t.cpu().numpy(), full_t[:, :5].cpu().numpy())
