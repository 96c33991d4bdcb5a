#!/usr/bin/env python
"""Benchmark of the relation-typed sparse hop path (MiniKG proof loop) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload kg_large] [--impl ours|reference]

A step is one training pass of the hop loop over one query batch: the forward of every hop
(the op of every frontier entry's messages, the concat-sum, the mass normalisation; then the
sum over rules) and its backward to the per-hop rule weights and the edge scores.  The metric
is edge-messages per second (GTEPS): the messages of all hops (frontier entries x their
out-edges, both directions) divided by the fwd+bwd step time.

Default workload: the 4,594,485-entity / 822-relation / 20,624,575-triple graph, 256 queries
x 4 rules x 2 hops, uncapped, frontier pruned to <= 0.5% of the entities
(``prune_sparse3d_active_entities`` at 22,972 entities), on the key-slab engine
(``slab_loop.SlabHopLoop``).  Under torchrun the same batch is destination-partitioned over
the ranks (rank k owns an entity range and walks only the messages into it; frontier
all-gather and row-sum all-reduce per hop over NCCL): strong scaling, ``value`` = the
step's messages over the slowest rank's time.  Workloads with a dense state (kg_small,
kg_mid, kg_skew) run the fused loop instead, as query-batch replicas under torchrun.

Prints one JSON line (rank 0).  ``--impl reference`` times the reference algorithm (the numpy
oracle port of the reference's CPU path) on the host cores instead.
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
SLAB_WORKLOADS = ("kg_large", "kg_web")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="kg_large")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="headline only (no kg_mid / capped / decode blocks)")
    ap.add_argument("--cpu-sample-queries", type=int, default=0, help="0: pick automatically")
    ap.add_argument("--queries", type=int, default=0, help="override the workload's query batch (profiling)")
    ap.add_argument("--engine", default="auto", choices=["auto", "slab", "fused", "sharded", "capped"],
                    help="auto: slab for the large graphs, fused otherwise; sharded: the capped sparse loop "
                         "destination-partitioned; capped: only the capped loops of the workload")
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


def timed(fn, steps, flush=None, stream_events=True):
    """Device time (ms) of each of ``steps`` calls, CUDA events around each, L2 flushed before."""
    import torch
    out = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record()
        fn()
        s1.record()
        s1.synchronize()
        out.append(s0.elapsed_time(s1))
    return out


def max_over_ranks(x: float, world: int, dev) -> float:
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU side
_W = {}


def _worker_init(head, rel, tail, E, R, heads, w_hops, scores, cap, topk_nodes=0):
    """Spawned worker: keeps the graph, its oracle CSR and the batch inputs."""
    sys.path.insert(0, str(ROOT))
    from oracle import fastlog_oracle as O
    _W.update(head=head, E=E, R=R, heads=heads, w_hops=w_hops, scores=scores, cap=cap, topk_nodes=topk_nodes,
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
    final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, cap=cap,
                                       topk_nodes=_W["topk_nodes"])
    seed = np.random.default_rng(0).standard_normal(final[0].shape[0]).astype(np.float32)
    O.proof_sum_backward(trace, (final[0], seed), w_hops, csr, mask, scores, B, L, E, R,
                         num_facts=_W["head"].shape[0])
    return sum(O.count_messages(tr["state"], csr, w_hops[k], L, E, R, cap) for k, tr in enumerate(trace))


def cpu_sample(kg, inp, queries: int, cap: int, topk_nodes: int = 0):
    """(messages, seconds) of the oracle on the first ``queries`` queries, one thread."""
    _worker_init(kg.head, kg.rel, kg.tail, kg.num_entities, kg.num_relations, inp.heads, inp.rule_weights,
                 inp.edge_scores, cap, topk_nodes)
    t0 = time.perf_counter()
    msgs = _oracle_queries(list(range(queries)))
    return msgs, time.perf_counter() - t0


def run_reference(a, wl, kg, rank, world):
    """The reference arm: the reference algorithm (oracle port) on all host cores, rank 0 only."""
    if rank != 0:
        return
    import multiprocessing as mp
    inp = hop_inputs(kg, wl.B, wl.L, wl.hops, seed=0)
    cores = min(os.cpu_count() or 1, 32)
    per = max(1, a.cpu_sample_queries or (1 if wl.name in SLAB_WORKLOADS else 2))
    n_q = min(wl.B, per * cores)
    chunks = [list(range(i, min(i + per, n_q))) for i in range(0, n_q, per)]
    # the oracle's CSR is built once here and inherited by forked workers (this process never
    # initialises CUDA, so forking is safe)
    _worker_init(kg.head, kg.rel, kg.tail, kg.num_entities, kg.num_relations, inp.heads, inp.rule_weights,
                 inp.edge_scores, wl.topk_edges, wl.topk_nodes)
    ctx = mp.get_context("fork")
    times, msgs_all = [], []
    with ctx.Pool(processes=min(cores, len(chunks))) as pool:
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
            "scaling": "strong" if wl.name in SLAB_WORKLOADS else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": wl.name, "queries_per_step": n_q, "rules": wl.L, "hops": wl.hops,
                       "entities": wl.E, "relations": wl.R, "triples": wl.T, "edge_cap": "uncapped",
                       "topk_nodes": wl.topk_nodes},
            "cpu_baseline": {"value": value, "unit": "GTEPS", "cores": min(cores, len(chunks)), "kind": "port",
                             "sample": f"{n_q} of {wl.B} queries per step, fwd+bwd of all {wl.hops} hops, numpy "
                                       f"oracle port of the reference CPU path in {len(chunks)} spawned processes"},
            "e2e": {"value": value, "unit": "GTEPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU: fused loop (dense state)
def fused_block(a, wl, kg, rank, world, local_rank):
    """The fused loop on a workload whose dense state fits (kg_mid shape): replayed CUDA-graph
    step, eager per-kernel roofline, e2e through the public API, max decode, capped row and the
    rule producer.  Returns the measurement dict (every rank)."""
    import torch
    import torch.distributed as dist
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.proof import ProofRunner

    dev = torch.device("cuda", local_rank)
    inp = hop_inputs(kg, wl.B, wl.L, wl.hops, seed=rank)
    g = DeviceGraph.from_triples(*(torch.from_numpy(x).to(dev) for x in (kg.head, kg.rel, kg.tail)),
                                 kg.num_entities, kg.num_relations)
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

    # compulsory bytes per hop: the pull of hop h reads the state entering hop h; a state is
    # charged dense (E x B L x 4 B) only where the fused loop holds it dense and it is dense,
    # sparse frontiers at 12 B per entry (8 B key, 4 B value)
    push_deg = g.push_degree()
    c = g.csr
    grp = ((c[8][1:] - c[8][:-1]) + (c[12][1:] - c[12][:-1])).to(torch.int64)
    BL = B * L
    dense = E * BL * 4
    graph_bytes, in_bytes, out_bytes = [], [], []
    acts = [runner.row_activity(h).bool() for h in range(K)]
    for h in range(K):
        act = acts[h]
        graph_bytes.append(int((push_deg[act] * 8 + grp[act] * 10 + 16).sum().item()))
    # entries of each state: read back from the active rows of the next hop (an upper bound of nnz)
    nnz_in = [B * L] + [int(acts[h + 1].sum().item()) * BL for h in range(K - 1)]
    for h in range(K):
        in_bytes.append(min(dense, nnz_in[h] * 12))
        out_bytes.append(min(dense, (nnz_in[h + 1] if h + 1 < K else E * BL) * 12))
    fwd_bytes = [graph_bytes[h] + in_bytes[h] + out_bytes[h] + BL * n * 4 for h in range(K)]
    bwd_bytes = [graph_bytes[h] + out_bytes[h] + 2 * in_bytes[h] + BL * n * 4 + T * 4 for h in range(K)]
    # decode: the same hops with packed 8-byte (value, arg) outputs
    dec_bytes = sum(graph_bytes[h] + in_bytes[h] + out_bytes[h] * 16 // 12 + BL * n * 4 for h in range(K))

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

    cg = runner.capture(heads, w_hops, out, msgs, G, scores, grad_w, grad_edge)
    for _ in range(max(3, a.warmup)):
        cg.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        step_ms = timed(cg.replay, a.steps, flush)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    del cg
    total_ms = max_over_ranks(float(sum(step_ms)), world, dev)
    M_all = M
    if world > 1:
        mm = torch.tensor([M], device=dev, dtype=torch.int64)
        dist.all_reduce(mm, op=dist.ReduceOp.SUM)
        M_all = int(mm.item())
    value = M_all * a.steps / (total_ms / 1e3) / 1e9

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
    e2e_graph = runner.capture(heads, w_hops, out, msgs, G, scores, grad_w, grad_edge,
                               host_inputs=copies_in, host_outputs=copies_out)
    for _ in range(max(3, a.warmup)):
        e2e_graph.replay()
    torch.cuda.synchronize()
    e2e_total = max_over_ranks(float(sum(timed(e2e_graph.replay, a.steps, flush))), world, dev)
    del e2e_graph
    e2e_value = M_all * a.steps / (e2e_total / 1e3) / 1e9

    res = {"workload": wl.name, "value": value, "ms_per_step": total_ms / a.steps, "messages_per_step": M_all,
           "messages_per_hop": msgs_host, "clocks": clocks.summary(),
           "eager_ms_per_step": statistics.mean(eager_ms),
           "e2e": {"value": e2e_value, "unit": "GTEPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                   "ms_per_step": e2e_total / a.steps,
                   "path": "ProofRunner.capture with host_inputs / host_outputs (pinned host buffers), replayed"}}
    if rank != 0 or world > 1:
        return res
    hbm, peak_kind = peaks()
    fwd_avg = [statistics.mean(x[h] for x in fwd_ms) for h in range(K)]
    bwd_avg = [statistics.mean(x[h] for x in bwd_ms) for h in range(K)]

    def kern(avg, byts):
        return {"ms_per_launch": sum(avg) / K, "bytes_per_launch": sum(byts) / K,
                "gbs": sum(byts) / (sum(avg) / 1e3) / 1e9, "ms_per_hop": avg, "bytes_per_hop": byts,
                "frac_per_hop": [b / (t / 1e3) / 1e9 / hbm for b, t in zip(byts, avg)]}
    kernels = {"fwd_pull_kernel": kern(fwd_avg, fwd_bytes), "bwd_pull_kernel": kern(bwd_avg, bwd_bytes)}
    dom = max(kernels, key=lambda k: kernels[k]["ms_per_launch"])
    traffic = None
    tfile = ROOT / "profiles" / f"traffic_{wl.name}.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(dom)
    res["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": kernels[dom]["gbs"], "peak": hbm, "unit": "GB/s",
                       "frac": kernels[dom]["gbs"] / hbm, "peak_kind": peak_kind, "traffic": traffic}
    res["kernels"] = kernels

    from minikg_dev_b200.proof import decode_max
    for _ in range(2):
        decode_max(g, heads, w_hops, 100, scores)
    torch.cuda.synchronize()
    dec_ms = statistics.mean(timed(lambda: decode_max(g, heads, w_hops, 100, scores), max(3, a.steps // 2), flush))
    res["decode"] = {"ms": dec_ms, "topk": 100, "gteps": M / (dec_ms / 1e3) / 1e9,
                     "roofline": {"bound": "hbm", "achieved": dec_bytes / (dec_ms / 1e3) / 1e9, "peak": hbm,
                                  "unit": "GB/s", "frac": dec_bytes / (dec_ms / 1e3) / 1e9 / hbm,
                                  "bytes": dec_bytes, "note": "all hops' compulsory bytes (packed 8-byte maxima) "
                                                              "over the whole decode time, top-k included"}}

    from minikg_dev_b200.proof import proof_scores
    cap = wl.capped_row

    def capped_step():
        wt = w_hops.detach().requires_grad_(True)
        sc = scores.detach().requires_grad_(True)
        out_c, msgs_c = proof_scores(g, heads, wt, sc, None, True, 1.0, 0.0, cap)
        (out_c * G).sum().backward()
        return msgs_c

    msgs_c = capped_step()
    M_cap = int(msgs_c.sum().item())
    for _ in range(2):
        capped_step()
    cap_ms = statistics.mean(timed(capped_step, max(3, a.steps // 2), flush))
    res["capped"] = {"edge_cap": cap, "ms_per_step": cap_ms, "messages_per_step": M_cap,
                     "gteps": M_cap / (cap_ms / 1e3) / 1e9,
                     "path": "fused loop with per-hop edge-cap take tables, fwd+bwd"}

    from minikg_dev_b200 import rules
    H = 64
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
        prod_ms[bw] = statistics.mean(timed(lambda: producer_step(bw), max(3, a.steps // 2)))
    res["rule_producer"] = {"ms_fwd": prod_ms[False], "ms_fwd_bwd": prod_ms[True], "queries": B,
                            "distinct_relations": int(torch.unique(q_rels).numel()), "emb_size": H, "channels": n}
    res["gpu_launches_per_step"] = 8 + 5 * K
    return res


def run_fused(a, wl, kg, rank, world, local_rank):
    """Fused-loop workload as the headline (query-batch replicas under torchrun)."""
    res = fused_block(a, wl, kg, rank, world, local_rank)
    if rank != 0:
        return
    B, L, K = wl.B, wl.L, wl.hops
    line = {"metric": METRIC, "value": res["value"], "unit": "GTEPS", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; shapes of the reference workload)",
            "config": {"workload": wl.name, "entities": kg.num_entities, "relations": kg.num_relations,
                       "triples": kg.num_triples, "queries_per_gpu": B, "global_queries": B * world, "rules": L,
                       "hops": K, "edge_cap": "uncapped",
                       "parallelism": f"query-batch x{world}" if world > 1 else "single GPU",
                       "l2": "flushed (256 MB write) before every timed step",
                       "step": "fwd+bwd of the fused loop replayed as one CUDA graph (ProofRunner.capture)",
                       "messages_per_step": res["messages_per_step"], "messages_per_hop": res["messages_per_hop"]},
            "e2e": res["e2e"], "gpu_launches": res["gpu_launches_per_step"] * a.steps if world == 1 else None,
            "clocks": res["clocks"]}
    for k in ("roofline", "kernels", "decode", "capped", "rule_producer"):
        if k in res:
            line[k] = res[k]
    if world == 1 and not a.no_cpu_baseline:
        inp = hop_inputs(kg, B, L, K, seed=0)
        q = a.cpu_sample_queries or 24
        msgs_cpu, secs = cpu_sample(kg, inp, q, wl.topk_edges)
        line["cpu_baseline"] = {"value": msgs_cpu / secs / 1e9, "unit": "GTEPS", "cores": 1, "kind": "port",
                                "sample": f"{q} of {B} queries, fwd+bwd of all {K} hops ({msgs_cpu} messages in "
                                          f"{secs:.1f} s), numpy oracle port of the reference CPU path"}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU: key-slab loop (large graphs)
def _seed_of(keys):
    """A fixed pseudo-random output gradient in [-1, 1) per result key (b * E + e)."""
    import torch
    h = (keys * 2654435761 + 40503) % 1000003
    return h.to(torch.float32) / 500001.5 - 1.0


def run_slab(a, wl, kg, rank, world, local_rank):
    import torch
    from minikg_dev_b200.graph import DeviceGraph
    from minikg_dev_b200.sharded import ShardSpec, message_in_counts, plan_dst_ranges
    from minikg_dev_b200.slab_loop import SlabEngine, SlabHopLoop, slab_proof_scores

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if kg is None:  # web-scale shapes: drawn on the device (every rank draws the same graph)
        from minikg_dev_b200.synth import KG, sample_graph_device
        head_d, rel_d, tail_d = sample_graph_device(wl.E, wl.R, wl.T, wl.gen, seed=0, device=dev)
        kg = KG(wl.name, wl.E, wl.R, np.broadcast_to(np.int8(0), (wl.T,)), np.empty(0), np.empty(0),
                meta={"generator": "device"})
    else:
        head_d, rel_d, tail_d = (torch.from_numpy(x).to(dev) for x in (kg.head, kg.rel, kg.tail))
    B = a.queries or wl.B
    L, K, E, T = wl.L, wl.hops, kg.num_entities, kg.num_triples
    n = 2 * kg.num_relations + 1
    inp = hop_inputs(kg, B, L, K, seed=0)
    g = DeviceGraph.from_triples(head_d, rel_d, tail_d, E, kg.num_relations)
    spec, bounds = None, [0, E]
    if world > 1:
        bounds = plan_dst_ranges(message_in_counts(head_d, tail_d, E), world)
        spec = ShardSpec(rank, world, bounds)
    del head_d, rel_d, tail_d
    eng = SlabEngine(g, bounds[rank], bounds[rank + 1]) if world > 1 else SlabEngine(g)
    heads = torch.from_numpy(inp.heads).to(dev)
    w_hops = torch.from_numpy(inp.rule_weights).to(dev)
    scores = torch.from_numpy(inp.edge_scores).to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def step():
        wt = w_hops.detach().requires_grad_(True)
        sc = scores.detach().requires_grad_(True)
        keys, vals, msgs = SlabHopLoop.apply(wt, sc, heads, eng, None, True, 1.0, wl.topk_nodes,
                                             wl.state_threshold, spec)
        (vals * _seed_of(keys)).sum().backward()
        return msgs

    for _ in range(max(3, a.warmup)):
        msgs = step()
    torch.cuda.synchronize()
    msgs_host = [int(x) for x in msgs.cpu()]
    M = sum(msgs_host)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        step_ms = timed(step, a.steps, flush)
    torch.cuda.synchronize()
    total_ms = max_over_ranks(float(sum(step_ms)), world, dev)
    value = M * a.steps / (total_ms / 1e3) / 1e9

    # kernels of this library launched by one step: its own and the CUB scans compiled into it
    # (torch's elementwise / CUB kernels, in torch's namespaces, not counted)
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    launches = sum(1 for e in prof.events()
                   if e.device_type == torch.autograd.DeviceType.CUDA
                   and ("mkg::" in e.name or e.name.startswith("void cub::")))

    # roofline: a traced step records events and algorithmic bytes around every expansion launch
    eng.trace = []
    step()
    torch.cuda.synchronize()
    trace, eng.trace = eng.trace, None
    kinds = {}
    for kind, evs, byts, tiles in trace:  # one entry per hop: its launches (groups of tiles)
        d = kinds.setdefault(kind, {"ms": [], "bytes": [], "tiles": tiles, "launches": 0})
        d["ms"].append(sum(e0.elapsed_time(e1) for e0, e1 in evs))
        d["bytes"].append(byts)
        d["launches"] += len(evs)

    # end to end through the public API (slab_proof_scores): the batch's query heads and rule
    # weights copied host -> device from pinned memory, the loss, message counts and rule-weight
    # gradient copied back; edge scores are resident model parameters (their gradient stays on
    # the device, as in training)
    heads_h = torch.from_numpy(inp.heads).pin_memory()
    w_h = torch.from_numpy(inp.rule_weights).pin_memory()
    loss_h = torch.empty(1, pin_memory=True)
    msgs_h = torch.empty(K, dtype=torch.int64, pin_memory=True)
    gw_h = torch.empty((K, B, L, n), pin_memory=True)
    heads_d = torch.empty_like(heads)
    w_d = torch.empty_like(w_hops)

    def e2e_step():
        heads_d.copy_(heads_h, non_blocking=True)
        w_d.copy_(w_h, non_blocking=True)
        wt = w_d.detach().requires_grad_(True)
        sc = scores.detach().requires_grad_(True)
        out, m = slab_proof_scores(eng, heads_d, wt, sc, None, True, 1.0, wl.topk_nodes, wl.state_threshold, spec)
        idx = out.indices()
        loss = (out.values() * _seed_of(idx[0] * E + idx[1])).sum()
        loss.backward()
        loss_h.copy_(loss.detach().reshape(1), non_blocking=True)
        msgs_h.copy_(m, non_blocking=True)
        gw_h.copy_(wt.grad, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_total = max_over_ranks(float(sum(timed(e2e_step, a.steps, flush))), world, dev)
    e2e_value = M * a.steps / (e2e_total / 1e3) / 1e9
    h2d = heads_h.numel() * 8 + w_h.numel() * 4
    d2h = 4 + msgs_h.numel() * 8 + gw_h.numel() * 4

    extras = {}
    if world == 1 and not a.no_extras:
        extras = slab_extras(a, wl, kg, g, eng, heads, w_hops, scores, flush, B)
    if rank != 0:
        return
    hbm, peak_kind = peaks()
    kernels = {}
    for kind, d in kinds.items():
        name = "slab_expand_kernel" if kind == "fwd" else "slab_expand_backward_kernel"
        # a hop runs one launch per group of destination tiles: its time is their sum, its bytes
        # the hop's
        kernels[name] = {"launches": d["launches"], "destination_tiles": d["tiles"],
                         "ms_per_launch": sum(d["ms"]) / d["launches"],
                         "ms_per_hop_mean": sum(d["ms"]) / len(d["ms"]),
                         "bytes_per_hop_mean": sum(d["bytes"]) / len(d["ms"]),
                         "gbs": sum(d["bytes"]) / (sum(d["ms"]) / 1e3) / 1e9, "ms_per_hop": d["ms"],
                         "bytes_per_hop": d["bytes"],
                         "frac_per_hop": [b / (t / 1e3) / 1e9 / hbm for b, t in zip(d["bytes"], d["ms"])]}
    dom = max(kernels, key=lambda k: sum(kernels[k]["ms_per_hop"]))
    traffic = None
    tfile = ROOT / "profiles" / f"traffic_{wl.name}.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(dom)
    line = {
        "metric": METRIC, "value": value, "unit": "GTEPS", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; shapes of the reference workload)",
        "config": {"workload": wl.name, "entities": E, "relations": kg.num_relations, "triples": T, "queries": B,
                   "rules": L, "hops": K, "edge_cap": "uncapped", "topk_nodes": wl.topk_nodes,
                   "engine": "key-slab hop loop (slab_loop.SlabHopLoop), fwd+bwd",
                   "parallelism": f"dst-partition x{world} (NCCL frontier all-gather, row-sum all-reduce)"
                   if world > 1 else "single GPU", "bounds": bounds if world > 1 else None,
                   "graph_generator": kg.meta.get("generator", "host"),
                   "l2": "flushed (256 MB write) before every timed step; graph lists and store exceed L2",
                   "messages_per_step": M, "messages_per_hop": msgs_host},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": kernels[dom]["gbs"], "peak": hbm, "unit": "GB/s",
                     "frac": kernels[dom]["gbs"] / hbm, "peak_kind": peak_kind, "traffic": traffic},
        "kernels": kernels,
        "e2e": {"value": e2e_value, "unit": "GTEPS", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_total / a.steps,
                "path": "slab_proof_scores (sparse [B, E] result) with pinned-host query heads and rule weights "
                        "in, loss / message counts / rule-weight gradient out"},
        "gpu_launches": launches * a.steps, "clocks": clocks.summary(),
    }
    line.update(extras)
    if world == 1 and not a.no_cpu_baseline:
        q = a.cpu_sample_queries or 32
        msgs_cpu, secs = cpu_sample(kg, inp, q, wl.topk_edges, wl.topk_nodes)
        line["cpu_baseline"] = {"value": msgs_cpu / secs / 1e9, "unit": "GTEPS", "cores": 1, "kind": "port",
                                "sample": f"{q} of {B} queries, fwd+bwd of all {K} hops ({msgs_cpu} messages in "
                                          f"{secs:.1f} s), numpy oracle port of the reference CPU path"}
    print(json.dumps(line), flush=True)


def slab_extras(a, wl, kg, g, eng, heads, w_hops, scores, flush, B):
    """Single-GPU extras beside the headline: the production-cap row of the same batch (sparse
    loop), its max decode, and the kg_mid fused block."""
    import torch
    from minikg_dev_b200.proof import decode_max_sparse
    from minikg_dev_b200.sparse_loop import sparse_proof_scores
    E = kg.num_entities
    out = {}
    cap = wl.capped_row

    def capped_step():
        wt = w_hops.detach().requires_grad_(True)
        sc = scores.detach().requires_grad_(True)
        o, m = sparse_proof_scores(g, heads, wt, sc, None, True, 1.0, cap, wl.topk_nodes)
        idx = o.indices()
        (o.values() * _seed_of(idx[0] * E + idx[1])).sum().backward()
        return m

    m = capped_step()
    M_cap = int(m.sum())
    ms = statistics.mean(timed(capped_step, 3, flush))
    out["capped"] = {"edge_cap": cap, "ms_per_step": ms, "messages_per_step": M_cap, "gteps": M_cap / ms / 1e6,
                     "path": "sparse hop loop (merged per-hop op, hash message store), fwd+bwd"}

    # the configuration's decode, uncapped: the max-aggregation loop on the key-slab store, top-100
    from minikg_dev_b200.slab_loop import slab_decode_max
    hbm, peak_kind = peaks()
    mlist = []
    slab_decode_max(eng, heads, w_hops, 100, scores, msgs_out=mlist)
    M_dec = int(torch.stack(mlist).sum())
    udec = lambda: slab_decode_max(eng, heads, w_hops, 100, scores)  # noqa: E731
    udms = statistics.mean(timed(udec, 3, flush))
    eng.trace = []
    udec()
    torch.cuda.synchronize()
    trace, eng.trace = eng.trace, None
    hop_ms = [sum(e0.elapsed_time(e1) for e0, e1 in evs) for _, evs, _, _ in trace]
    hop_bytes = [byts for _, _, byts, _ in trace]
    gbs = sum(hop_bytes) / (sum(hop_ms) / 1e3) / 1e9
    out["decode_uncapped"] = {
        "ms": udms, "topk": 100, "edge_cap": "uncapped", "messages": M_dec, "gteps": M_dec / udms / 1e6,
        "path": "slab_loop.slab_decode_max (atomicMax key slab, ordered row sums, max over rules, device top-k)",
        "roofline": {"bound": "hbm", "kernel": "slab_expand_kernel (max mode)", "achieved": gbs, "peak": hbm,
                     "unit": "GB/s", "frac": gbs / hbm, "peak_kind": peak_kind, "ms_per_hop": hop_ms,
                     "bytes_per_hop": hop_bytes}}

    # the production-cap decode of the same batch: the max-aggregation sparse loop, top-100
    dec = lambda: decode_max_sparse(g, heads, w_hops, 100, scores, cap=cap)  # noqa: E731
    dec()
    dms = statistics.mean(timed(dec, 3, flush))
    out["decode"] = {"ms": dms, "topk": 100, "edge_cap": cap, "gteps": M_cap / dms / 1e6,
                     "path": "proof.decode_max_sparse (max op with argmax, ordered row sums, device top-k)"}

    # the mid-size graph's fused loop (dense state), its decode, capped row and rule producer
    mid = WORKLOADS["kg_mid"]
    mid_kg = workload_graph("kg_mid", seed=0)
    res = fused_block(a, mid, mid_kg, 0, 1, 0)
    out["kg_mid"] = res
    return out


# ----------------------------------------------------------------------------- GPU: capped sparse loop, sharded
def run_sharded(a, wl, kg, rank, world, local_rank):
    """The destination-partitioned capped sparse loop (production cap of the workload)."""
    import torch
    import torch.distributed as dist
    from minikg_dev_b200 import sharded as S
    from minikg_dev_b200.graph import DeviceGraph

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if kg is None:
        from minikg_dev_b200.synth import KG, sample_graph_device
        head_d, rel_d, tail_d = sample_graph_device(wl.E, wl.R, wl.T, wl.gen, seed=0, device=dev)
        kg = KG(wl.name, wl.E, wl.R, np.broadcast_to(np.int8(0), (wl.T,)), np.empty(0), np.empty(0),
                meta={"generator": "device"})
    else:
        head_d, rel_d, tail_d = (torch.from_numpy(x).to(dev) for x in (kg.head, kg.rel, kg.tail))
    B, L, K, E, T = wl.B, wl.L, wl.hops, kg.num_entities, kg.num_triples
    cap = wl.capped_row
    inp = hop_inputs(kg, B, L, K, seed=0)
    g = DeviceGraph.from_triples(head_d, rel_d, tail_d, E, kg.num_relations)
    bounds = S.plan_dst_ranges(S.message_in_counts(head_d, tail_d, E), world)
    del head_d, rel_d, tail_d
    spec = S.ShardSpec(rank, world, bounds)
    heads = torch.from_numpy(inp.heads).to(dev)
    w0 = torch.from_numpy(inp.rule_weights).to(dev)
    s0 = torch.from_numpy(inp.edge_scores).to(dev)
    counter = S.message_counter(g, cap)

    def step():
        wt = w0.detach().requires_grad_(True)
        sc = s0.detach().requires_grad_(True)
        hop = S.cuda_hop_fn(g, None, S.replicated(sc, spec.group), cap, True, 1.0)
        msgs = []
        keys, vals = S.sharded_proof_scores(spec, hop, heads, wt, E, threshold=wl.state_threshold,
                                            topk_nodes=wl.topk_nodes, msg_counter=counter, msgs_out=msgs)
        (vals * _seed_of(keys)).sum().backward()
        return torch.stack(msgs)

    for _ in range(max(3, a.warmup)):
        msgs = step()
    M = int(msgs.sum().item())
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        step_ms = timed(step, a.steps)
    total_ms = max_over_ranks(float(sum(step_ms)), world, dev)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": M * a.steps / (total_ms / 1e3) / 1e9, "unit": "GTEPS",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": total_ms / a.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "engine": "sharded capped sparse loop",
            "config": {"workload": wl.name, "entities": E, "relations": kg.num_relations, "triples": T,
                       "queries": B, "rules": L, "hops": K, "edge_cap": cap,
                       "graph_generator": kg.meta.get("generator", "host"),
                       "parallelism": f"dst-partition x{world}", "bounds": bounds},
            "messages_per_step": M, "clocks": clocks.summary()}), flush=True)


def main():
    a = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[a.workload]
    engine = a.engine
    if engine == "auto":
        engine = "slab" if wl.name in SLAB_WORKLOADS else "fused"
    # graphs above 5e7 facts are drawn on the GPU by the GPU engines themselves
    host_graph = wl.T <= 50_000_000 or a.impl == "reference"
    if a.impl == "reference" and rank != 0:
        return
    kg = workload_graph(a.workload, seed=0) if host_graph else None
    if a.impl == "reference":
        run_reference(a, wl, kg, rank, world)
        return
    distributed = world > 1 or engine == "sharded"
    if distributed:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29531")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), rank=rank, world_size=world,
                                device_id=torch.device("cuda", local_rank))
    try:
        if engine == "slab":
            run_slab(a, wl, kg, rank, world, local_rank)
        elif engine == "sharded":
            run_sharded(a, wl, kg, rank, world, local_rank)
        else:
            run_fused(a, wl, kg, rank, world, local_rank)
    finally:
        if distributed:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
