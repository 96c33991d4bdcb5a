#!/usr/bin/env python
"""Benchmark of the relation-typed sparse hop path (MiniKG proof loop) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload kg_mid] [--impl ours|reference]

A step is one training pass of the hop loop over one query batch: the forward of every
hop (op + concat + mass normalisation, then the sum over rules) and its backward to the
per-hop rule weights and the edge scores, on the 17,050-entity / 51-relation /
206,205-triple synthetic graph with 256 queries x 3 rules x 3 hops, uncapped, captured once
as a CUDA graph and replayed (``ProofRunner.capture``; the eager step is reported beside it and
supplies the per-kernel roofline times).  The metric is edge-messages per second (GTEPS): the
messages of all hops (frontier entries x their taken out-edges, both directions) divided by the
fwd+bwd step time.  Under torchrun
every rank runs its own 256 queries on a replica of the graph (query-batch sharding, weak
scaling, no collective in the data path); ``value`` sums all ranks' messages over the
slowest rank's time.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference algorithm
(the numpy oracle port of the reference's CPU path) on the host cores instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from minikg_dev_b200.synth import WORKLOADS, hop_inputs, workload_graph  # noqa: E402

METRIC = "GTEPS (edge-msgs/s) per hop fwd+bwd & argmax decode; % of HBM roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="kg_mid")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-queries", type=int, default=0, help="0: pick automatically")
    ap.add_argument("--engine", default="fused", choices=["fused", "sharded", "capped"],
                    help="sharded: destination-partitioned capped hop loop (kg_large / kg_web shapes); "
                         "capped: only the capped sparse loop of the workload (for profiling)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers
def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU side
_W = {}


def _worker_init(head, rel, tail, E, R, heads, w_hops, scores, cap):
    """Spawned worker: keeps the graph, its oracle CSR and the batch inputs."""
    sys.path.insert(0, str(ROOT))
    from oracle import fastlog_oracle as O
    _W.update(head=head, E=E, R=R, heads=heads, w_hops=w_hops, scores=scores, cap=cap,
              csr=O.build_csr_structure(head, tail, rel, E))


def _oracle_queries(query_ids):
    """One fwd+bwd of the hop loop on a query subset with the numpy oracle; returns messages."""
    from oracle import fastlog_oracle as O
    q = np.asarray(query_ids, np.int64)
    heads = _W["heads"][q]
    w_hops = np.ascontiguousarray(_W["w_hops"][:, q])
    E, R, csr, scores, cap = _W["E"], _W["R"], _W["csr"], _W["scores"], _W["cap"]
    B, L = heads.shape[0], w_hops.shape[2]
    mask = np.ones(_W["head"].shape[0], bool)
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, cap=cap)
    seed = np.random.default_rng(0).standard_normal(final[0].shape[0]).astype(np.float32)
    O.proof_sum_backward(trace, (final[0], seed), w_hops, csr, mask, scores, B, L, E, R,
                         num_facts=_W["head"].shape[0])
    return sum(O.count_messages(tr["state"], csr, w_hops[k], L, E, R, cap) for k, tr in enumerate(trace))


def cpu_sample(kg, inp, queries: int, cap: int):
    """(messages, seconds) of the oracle on the first ``queries`` queries, one thread."""
    _worker_init(kg.head, kg.rel, kg.tail, kg.num_entities, kg.num_relations, inp.heads, inp.rule_weights,
                 inp.edge_scores, cap)
    t0 = time.perf_counter()
    msgs = _oracle_queries(list(range(queries)))
    return msgs, time.perf_counter() - t0


def run_reference(a, wl, kg, rank, world):
    """The reference arm: the reference algorithm (oracle port) on all host cores, rank 0 only."""
    if rank != 0:
        return
    import multiprocessing as mp
    inp = hop_inputs(kg, wl.B, wl.L, wl.hops, seed=0)
    cores = os.cpu_count() or 1
    per = max(1, a.cpu_sample_queries or 2)
    n_q = min(wl.B, per * cores)
    chunks = [list(range(i, min(i + per, n_q))) for i in range(0, n_q, per)]
    ctx = mp.get_context("spawn")
    times, msgs_all = [], []
    with ctx.Pool(processes=min(cores, len(chunks)), initializer=_worker_init,
                  initargs=(kg.head, kg.rel, kg.tail, kg.num_entities, kg.num_relations, inp.heads,
                            inp.rule_weights, inp.edge_scores, wl.topk_edges)) as pool:
        for it in range(a.warmup + a.steps):
            t0 = time.perf_counter()
            msgs = sum(pool.map(_oracle_queries, chunks))
            dt = time.perf_counter() - t0
            if it >= a.warmup:
                times.append(dt)
                msgs_all.append(msgs)
    value = sum(msgs_all) / sum(times) / 1e9
    line = {"metric": METRIC, "value": value, "unit": "GTEPS", "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": 1e3 * statistics.mean(times), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": wl.name, "queries_per_step": n_q, "rules": wl.L, "hops": wl.hops,
                       "entities": wl.E, "relations": wl.R, "triples": wl.T, "edge_cap": "uncapped"},
            "cpu_baseline": {"value": value, "unit": "GTEPS", "cores": min(cores, len(chunks)), "kind": "port",
                             "sample": f"{n_q} of {wl.B} queries per step, fwd+bwd of all {wl.hops} hops, numpy "
                                       f"oracle port of the reference CPU path in {len(chunks)} spawned processes"},
            "e2e": {"value": value, "unit": "GTEPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU side
def run_ours(a, wl, kg, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import ProofRunner

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    inp = hop_inputs(kg, wl.B, wl.L, wl.hops, seed=rank)
    head = torch.from_numpy(kg.head).to(dev)
    rel = torch.from_numpy(kg.rel).to(dev)
    tail = torch.from_numpy(kg.tail).to(dev)
    g = DeviceGraph.from_triples(head, rel, tail, kg.num_entities, kg.num_relations)
    g.adjacency()
    B, L, K, E, T = wl.B, wl.L, wl.hops, kg.num_entities, kg.num_triples
    n = 2 * kg.num_relations + 1
    heads = torch.from_numpy(inp.heads).to(dev)
    w_hops = torch.from_numpy(inp.rule_weights).to(dev)
    scores = torch.from_numpy(inp.edge_scores).to(dev)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    G = torch.randn((B, E), device=dev, generator=gen)  # d loss / d scores on the result's keys
    runner = ProofRunner(g, B, L, K)
    out = torch.empty((B, E), device=dev)
    msgs = torch.zeros(K, dtype=torch.int64, device=dev)
    grad_w = torch.empty((K, B, L, n), device=dev)
    grad_edge = torch.empty(T, device=dev)
    ev_f = [torch.cuda.Event(enable_timing=True) for _ in range(2 * K)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(2 * K)]
    for e in ev_f + ev_b:
        e.record()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # > 126 MB L2

    def step(events=True):
        g.set_edge_factor(None, scores, True, 1.0)
        runner.forward(heads, w_hops, out, msgs, ev_f if events else None)
        runner.backward(G, None, scores, True, 1.0, True, grad_w, grad_edge, ev_b if events else None)

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    from minikg_dev_b200 import _native
    _native.raise_device_errors(dev)
    msgs_host = [int(x) for x in msgs.cpu()]
    M = sum(msgs_host)

    # compulsory bytes per hop (pull of hop h reads the state entering hop h)
    push_deg = g.push_degree()
    c = g.csr
    grp = ((c[8][1:] - c[8][:-1]) + (c[12][1:] - c[12][:-1])).to(torch.int64)
    graph_bytes = []
    for h in range(K):
        act = runner.row_activity(h).bool()
        graph_bytes.append(int((push_deg[act] * 8 + grp[act] * 10 + 16).sum().item()))
    BL = B * L
    dense = E * BL * 4
    fwd_bytes = [gb + 2 * dense + BL * n * 4 for gb in graph_bytes]
    bwd_bytes = [gb + 3 * dense + BL * n * 4 + T * 4 for gb in graph_bytes]

    # eager steps: the library records events around every pull kernel (the roofline's
    # per-launch times; events cannot be timed inside a CUDA graph)
    torch.cuda.synchronize()
    eager_ms, fwd_ms, bwd_ms = [], [], []
    for _ in range(a.steps):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        step()
        s1.record()
        s1.synchronize()
        eager_ms.append(s0.elapsed_time(s1))
        fwd_ms.append([ev_f[2 * h].elapsed_time(ev_f[2 * h + 1]) for h in range(K)])
        bwd_ms.append([ev_b[2 * h].elapsed_time(ev_b[2 * h + 1]) for h in range(K)])

    # the headline: the same step (edge-factor refresh, forward, backward) captured once as a
    # CUDA graph (ProofRunner.capture, public API) and replayed, L2 flushed before every step
    cg = runner.capture(heads, w_hops, out, msgs, G, scores, grad_w, grad_edge)
    for _ in range(max(3, a.warmup)):
        cg.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    step_ms = []
    with ClockSampler(local_rank) as clocks:
        for _ in range(a.steps):
            flush.zero_()
            s0 = torch.cuda.Event(enable_timing=True)
            s1 = torch.cuda.Event(enable_timing=True)
            s0.record()
            cg.replay()
            s1.record()
            s1.synchronize()
            step_ms.append(s0.elapsed_time(s1))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    del cg
    total_ms = float(sum(step_ms))
    M_all = M
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        mm = torch.tensor([M], device=dev, dtype=torch.int64)
        dist.all_reduce(mm, op=dist.ReduceOp.SUM)
        M_all = int(mm.item())
    value = M_all * a.steps / (total_ms / 1e3) / 1e9

    # end to end through the public API, host buffers, copies inside the timed region: the
    # step captured with its host copies (ProofRunner.capture with host_inputs / host_outputs)
    # and replayed; the same step with the copies launched eagerly is reported beside it.  The
    # step's results read back: message counts, rule-weight and edge-score gradients.
    heads_h = torch.from_numpy(inp.heads).pin_memory()
    w_h = torch.from_numpy(inp.rule_weights).pin_memory()
    scores_h = torch.from_numpy(inp.edge_scores).pin_memory()
    msgs_h = torch.empty(msgs.shape, dtype=torch.int64, pin_memory=True)
    gw_h = torch.empty((K, B, L, n), pin_memory=True)
    ge_h = torch.empty(T, pin_memory=True)
    h2d = heads_h.numel() * 8 + w_h.numel() * 4 + scores_h.numel() * 4
    d2h = msgs_h.numel() * 8 + gw_h.numel() * 4 + ge_h.numel() * 4
    copies_in = [(heads, heads_h), (w_hops, w_h), (scores, scores_h)]
    copies_out = [(msgs_h, msgs), (gw_h, grad_w), (ge_h, grad_edge)]

    def e2e_eager_step():
        for d, h in copies_in:
            d.copy_(h, non_blocking=True)
        g.set_edge_factor(None, scores, True, 1.0)
        runner.forward(heads, w_hops, out, msgs)
        runner.backward(G, None, scores, True, 1.0, True, grad_w, grad_edge)
        for h, d in copies_out:
            h.copy_(d, non_blocking=True)

    e2e_graph = runner.capture(heads, w_hops, out, msgs, G, scores, grad_w, grad_edge,
                               host_inputs=copies_in, host_outputs=copies_out)

    def time_e2e(fn):
        for _ in range(max(3, a.warmup)):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        times = []
        for _ in range(a.steps):
            flush.zero_()
            s0 = torch.cuda.Event(enable_timing=True)
            s1 = torch.cuda.Event(enable_timing=True)
            s0.record()
            fn()
            s1.record()
            s1.synchronize()
            times.append(s0.elapsed_time(s1))
        total = float(sum(times))
        if world > 1:
            t = torch.tensor([total], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total = float(t.item())
        return total

    e2e_total = time_e2e(e2e_graph.replay)
    e2e_eager_total = time_e2e(e2e_eager_step)
    del e2e_graph
    e2e_value = M_all * a.steps / (e2e_total / 1e3) / 1e9
    e2e_eager_value = M_all * a.steps / (e2e_eager_total / 1e3) / 1e9

    # max-argmax decode (forward only) of the same batch, top-100 answers per query
    from minikg_dev_b200.proof import decode_max
    for _ in range(2):
        decode_max(g, heads, w_hops, 100, scores)
    torch.cuda.synchronize()
    dec_ms = []
    for _ in range(max(3, a.steps // 2)):
        flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        decode_max(g, heads, w_hops, 100, scores)
        s1.record()
        s1.synchronize()
        dec_ms.append(s0.elapsed_time(s1))

    # capped row: the same batch with the reference's production edge cap of 100, forward +
    # backward, on the fused loop (per-hop take tables of the capped rows; the path
    # kernel_sparse_scores takes) and, for comparison, on the sparse loop (per-hop op with the
    # 256-bucket cap and merged outputs, device normalisation, written-out backward)
    from minikg_dev_b200.proof import proof_scores
    from minikg_dev_b200.sparse_loop import sparse_proof_scores
    cap = 100

    def capped_step():
        wt = w_hops.detach().requires_grad_(True)
        sc = scores.detach().requires_grad_(True)
        out_c, msgs_c = proof_scores(g, heads, wt, sc, None, True, 1.0, 0.0, cap)
        (out_c * G).sum().backward()
        return msgs_c

    def capped_sparse_step():
        wt = w_hops.detach().requires_grad_(True)
        sc = scores.detach().requires_grad_(True)
        out_c, msgs_c = sparse_proof_scores(g, heads, wt, sc, None, True, 1.0, cap, 0)
        oi = out_c.indices()
        (out_c.values() * G[oi[0], oi[1]]).sum().backward()
        return msgs_c

    def time_steps(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, a.steps // 2)):
            flush.zero_()
            s0 = torch.cuda.Event(enable_timing=True)
            s1 = torch.cuda.Event(enable_timing=True)
            s0.record()
            fn()
            s1.record()
            s1.synchronize()
            ts.append(s0.elapsed_time(s1))
        return ts

    msgs_c = capped_step()
    M_cap = int(msgs_c.sum().item())
    cap_ms = time_steps(capped_step)
    cap_sparse_ms = time_steps(capped_sparse_step)

    # rule-weight producer (per-rule BiLSTM -> linear -> per-hop softmax) for the same batch's
    # target relations: random-init parameters of the reference model's shapes, fwd and fwd+bwd
    from minikg_dev_b200 import rules
    H = 48 if wl.name == "kg_small" else 64
    torch.manual_seed(rank)
    pm = torch.nn.Module()
    pm.emb = torch.nn.Parameter(torch.randn(n, H) * 0.5)
    pm.lstm = torch.nn.ModuleList(torch.nn.LSTM(H, H, 1, bidirectional=True) for _ in range(L))
    pm.linear = torch.nn.Linear(2 * H, n)
    pm.step, pm.relation_count, pm.tau_1 = K, kg.num_relations, 1.0
    pm.to(dev)
    q_rels = torch.randint(0, kg.num_relations, (B,), device=dev)
    Gw = torch.randn(K, B, L, n, device=dev)

    def producer_step(backward: bool):
        pm.zero_grad(set_to_none=True)
        w = rules.rule_weights(pm, q_rels)
        if backward:
            (w * Gw).sum().backward()

    prod_ms = {}
    for bw in (False, True):
        for _ in range(3):
            producer_step(bw)
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, a.steps // 2)):
            s0 = torch.cuda.Event(enable_timing=True)
            s1 = torch.cuda.Event(enable_timing=True)
            s0.record()
            producer_step(bw)
            s1.record()
            s1.synchronize()
            ts.append(s0.elapsed_time(s1))
        prod_ms[bw] = statistics.mean(ts)

    if rank != 0:
        return
    hbm, peak_kind = peaks()
    fwd_avg = [statistics.mean(x[h] for x in fwd_ms) for h in range(K)]
    bwd_avg = [statistics.mean(x[h] for x in bwd_ms) for h in range(K)]
    kernels = {
        "fwd_pull_kernel": {"ms_per_launch": sum(fwd_avg) / K, "bytes_per_launch": sum(fwd_bytes) / K,
                            "gbs": sum(fwd_bytes) / (sum(fwd_avg) / 1e3) / 1e9, "ms_per_hop": fwd_avg},
        "bwd_pull_kernel": {"ms_per_launch": sum(bwd_avg) / K, "bytes_per_launch": sum(bwd_bytes) / K,
                            "gbs": sum(bwd_bytes) / (sum(bwd_avg) / 1e3) / 1e9, "ms_per_hop": bwd_avg},
    }
    dom = max(kernels, key=lambda k: kernels[k]["ms_per_launch"])
    traffic = None
    tfile = ROOT / "profiles" / f"traffic_{wl.name}.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(dom)
    line = {
        "metric": METRIC, "value": value, "unit": "GTEPS", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; shapes of the reference workload)",
        "config": {"workload": wl.name, "entities": E, "relations": kg.num_relations, "triples": T,
                   "queries_per_gpu": B, "global_queries": B * world, "rules": L, "hops": K,
                   "edge_cap": "uncapped", "parallelism": f"query-batch x{world}" if world > 1 else "single GPU",
                   "l2": "flushed (256 MB write) before every timed step",
                   "step": "fwd+bwd of the fused loop replayed as one CUDA graph (ProofRunner.capture)",
                   "messages_per_step": M_all, "messages_per_hop": msgs_host},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": kernels[dom]["gbs"], "peak": hbm, "unit": "GB/s",
                     "frac": kernels[dom]["gbs"] / hbm, "peak_kind": peak_kind, "traffic": traffic},
        "kernels": kernels,
        "decode": {"ms": statistics.mean(dec_ms), "topk": 100,
                   "gteps": M / (statistics.mean(dec_ms) / 1e3) / 1e9},
        "eager": {"ms_per_step": statistics.mean(eager_ms), "gteps": M / (statistics.mean(eager_ms) / 1e3) / 1e9,
                  "note": "the same step launched eagerly (per-kernel events for the roofline)"},
        "capped": {"edge_cap": cap, "ms_per_step": statistics.mean(cap_ms), "messages_per_step": M_cap,
                   "gteps": M_cap / (statistics.mean(cap_ms) / 1e3) / 1e9,
                   "path": "fused loop with per-hop edge-cap take tables (the path kernel_sparse_scores "
                           "takes for caps <= 255), fwd+bwd",
                   "sparse_loop_ms_per_step": statistics.mean(cap_sparse_ms)},
        "rule_producer": {"ms_fwd": prod_ms[False], "ms_fwd_bwd": prod_ms[True], "queries": B,
                          "distinct_relations": int(torch.unique(q_rels).numel()), "emb_size": H, "channels": n,
                          "path": "per-relation BiLSTM + SGEMM linear layer + per-hop softmax (rules.rule_weights),"
                                  " random-init parameters of the reference model's shapes"},
        "e2e": {"value": e2e_value, "unit": "GTEPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_total / a.steps,
                "path": "ProofRunner.capture with host_inputs / host_outputs (pinned host buffers), replayed",
                "eager_value": e2e_eager_value, "eager_ms_per_step": e2e_eager_total / a.steps},
        "gpu_launches": (8 + 5 * K) * a.steps,
        "clocks": clocks.summary(),
    }
    if world == 1 and not a.no_cpu_baseline:
        q = a.cpu_sample_queries or 24
        msgs_cpu, secs = cpu_sample(kg, inp, q, wl.topk_edges)
        line["cpu_baseline"] = {"value": msgs_cpu / secs / 1e9, "unit": "GTEPS", "cores": 1, "kind": "port",
                                "sample": f"{q} of {B} queries, fwd+bwd of all {K} hops ({msgs_cpu} messages in "
                                          f"{secs:.1f} s), numpy oracle port of the reference CPU path"}
    print(json.dumps(line), flush=True)


def run_sharded(a, wl, kg, rank, world, local_rank):
    """The destination-partitioned capped hop loop: every rank holds the whole CSR and owns an
    entity range; the query batch is the workload's (strong scaling over ranks)."""
    import torch
    import torch.distributed as dist
    from minikg_dev_b200 import sharded as S
    from minikg_dev_b200.graph import DeviceGraph

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if kg is None:  # web-scale shapes: drawn on the device (every rank draws the same graph)
        from minikg_dev_b200.synth import KG, sample_graph_device
        head_d, rel_d, tail_d = sample_graph_device(wl.E, wl.R, wl.T, wl.gen, seed=0, device=dev)
        kg = KG(wl.name, wl.E, wl.R, np.broadcast_to(np.int8(0), (wl.T,)), np.empty(0), np.empty(0),
                meta={"generator": "device"})
    else:
        head_d, rel_d, tail_d = (torch.from_numpy(a).to(dev) for a in (kg.head, kg.rel, kg.tail))
    B, L, K, E, T = wl.B, wl.L, wl.hops, kg.num_entities, kg.num_triples
    inp = hop_inputs(kg, B, L, K, seed=0)
    g = DeviceGraph.from_triples(head_d, rel_d, tail_d, E, kg.num_relations)
    bounds = S.plan_dst_ranges(S.message_in_counts(head_d, tail_d, E), world)
    del head_d, rel_d, tail_d
    spec = S.ShardSpec(rank, world, bounds)
    heads = torch.from_numpy(inp.heads).to(dev)
    w0 = torch.from_numpy(inp.rule_weights).to(dev)
    s0 = torch.from_numpy(inp.edge_scores).to(dev)
    counter = S.message_counter(g, wl.topk_edges)
    seed = torch.randn(B * E, device=dev, generator=torch.Generator(device=dev).manual_seed(1234))

    def step():
        wt = w0.detach().requires_grad_(True)
        sc = s0.detach().requires_grad_(True)
        hop = S.cuda_hop_fn(g, None, S.replicated(sc, spec.group), wl.topk_edges, True, 1.0)
        msgs = []
        keys, vals = S.sharded_proof_scores(spec, hop, heads, wt, E, threshold=wl.state_threshold,
                                            topk_nodes=wl.topk_nodes, msg_counter=counter, msgs_out=msgs)
        (vals * seed[keys]).sum().backward()
        return torch.stack(msgs), wt.grad, sc.grad

    for _ in range(max(3, a.warmup)):
        msgs, _, _ = step()
    M = int(msgs.sum().item())
    dist.barrier()
    torch.cuda.synchronize()
    step_ms = []
    with ClockSampler(local_rank) as clocks:
        for _ in range(a.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            e1.synchronize()
            step_ms.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([float(sum(step_ms))], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": M * a.steps / (total_ms / 1e3) / 1e9, "unit": "GTEPS",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": total_ms / a.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "engine": "sharded",
            "config": {"workload": wl.name, "entities": E, "relations": kg.num_relations, "triples": T,
                       "queries": B, "rules": L, "hops": K, "topk_edges": wl.topk_edges,
                       "graph_generator": kg.meta.get("generator", "host"),
                       "parallelism": f"dst-partition x{world}", "bounds": bounds,
                       "l2": "state and inputs exceed L2"},
            "messages_per_step": M, "clocks": clocks.summary()}), flush=True)


def run_capped(a, wl, kg):
    """Only the capped (cap 100) hop loop, fwd+bwd, on the fused loop and on the sparse loop."""
    import torch
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.sparse_loop import sparse_proof_scores
    dev = torch.device("cuda", 0)
    B, L, K, E = wl.B, wl.L, wl.hops, kg.num_entities
    inp = hop_inputs(kg, B, L, K, seed=0)
    g = DeviceGraph.from_triples(torch.from_numpy(kg.head).to(dev), torch.from_numpy(kg.rel).to(dev),
                                 torch.from_numpy(kg.tail).to(dev), E, kg.num_relations)
    heads = torch.from_numpy(inp.heads).to(dev)
    w0 = torch.from_numpy(inp.rule_weights).to(dev)
    s0 = torch.from_numpy(inp.edge_scores).to(dev)
    G = torch.randn((B, E), device=dev, generator=torch.Generator(device=dev).manual_seed(1234))

    from minikg_dev_b200.proof import proof_scores

    def fused_step():
        wt = w0.detach().requires_grad_(True)
        sc = s0.detach().requires_grad_(True)
        out, msgs = proof_scores(g, heads, wt, sc, None, True, 1.0, 0.0, 100)
        (out * G).sum().backward()
        return msgs

    def sparse_step():
        wt = w0.detach().requires_grad_(True)
        sc = s0.detach().requires_grad_(True)
        out, msgs = sparse_proof_scores(g, heads, wt, sc, None, True, 1.0, 100, 0)
        oi = out.indices()
        (out.values() * G[oi[0], oi[1]]).sum().backward()
        return msgs

    res = {}
    for name, step in (("fused", fused_step), ("sparse_loop", sparse_step)):
        for _ in range(max(3, a.warmup)):
            msgs = step()
        torch.cuda.synchronize()
        ms = []
        for _ in range(a.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            e1.synchronize()
            ms.append(e0.elapsed_time(e1))
        M = int(msgs.sum().item())
        res[name] = {"messages_per_step": M, "ms_per_step": statistics.mean(ms),
                     "gteps": M / (statistics.mean(ms) / 1e3) / 1e9}
    print(json.dumps({"engine": "capped", "workload": wl.name, "edge_cap": 100, **res}))


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[a.workload]
    # graphs above 5e7 facts are drawn on the GPU by the sharded engine itself
    kg = None if (a.engine == "sharded" and wl.T > 50_000_000) else workload_graph(a.workload, seed=0)
    if a.impl == "reference":
        run_reference(a, wl, kg, rank, world)
        return
    if a.engine == "capped":
        run_capped(a, wl, kg)
        return
    distributed = world > 1 or a.engine == "sharded"
    if distributed:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29531")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), rank=rank, world_size=world,
                                device_id=torch.device("cuda", local_rank))
    try:
        if a.engine == "sharded":
            run_sharded(a, wl, kg, rank, world, local_rank)
        else:
            run_ours(a, wl, kg, rank, world, local_rank)
    finally:
        if distributed:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
