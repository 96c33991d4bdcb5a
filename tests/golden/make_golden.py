"""Golden vectors for the relation-typed sparse hop, produced by the reference's own code.

Run where a checkout of the reference exists (it does not travel):

    python tests/golden/make_golden.py --ref <path of the reference checkout>

The reference's hop op (``FastLogFunctionSparse3DTopK``, fastlog_kernel.py:900-1107)
calls a CUDA extension.  With no GPU here, the extension object it loads is replaced
by ``_CpuExtension`` below, which answers each CUDA entry point with the reference's
own CPU code:

* forward: ``_expand_sparse3d_direction_cpu`` (fastlog_kernel.py:1523-1634) run twice
  per direction, once with the real ``col_ind`` (destinations) and once with
  ``arange(T)`` in its place (CSR positions, hence ``meta_edge = order[pos]``); the
  per-position factor is ``bool(mask) * score`` as in fastlog.cu:2303-2309;
* sum backward: ``FastLogFunctionSparse3DCPU.backward`` (fastlog_kernel.py:1681-1720);
* argmax backward: a five-line restatement of fastlog.cu:2646-2676 (scatter of the
  aligned raw gradient) plus the reference's identity-channel gather.

Everything else — coalescing, argmax tie-breaking, the edge-score gradient, the bridge
reducers, ``normalize_sparse3d``, ``kernel_sparse_scores``, ``sparse3d_max`` /
``norm_sp_3d_max``, bound and decode ordering — is the reference's code, unchanged.
Inputs use strictly positive edge factors so the CPU expansion (which drops zero
factors) and the CUDA fill (which keeps them) emit the same messages.
"""
from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from minikg_dev_b200.synth import sample_graph, softmax_f32  # noqa: E402

UNCAPPED = 1 << 60


def import_reference(ref: str):
    stub = types.ModuleType("torch_scatter")

    def _missing(*_a, **_k):
        raise RuntimeError("torch_scatter is not installed; off the hop path")

    stub.scatter_max = stub.scatter_sum = stub.scatter_add = stub.scatter = _missing
    sys.modules.setdefault("torch_scatter", stub)
    for p in (ref, os.path.join(ref, "src")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import fastlog_kernel.fastlog_kernel as fk  # noqa: E402
    import model_mmDRUM_kernel_sp as mm  # noqa: E402
    import drum  # noqa: E402
    import proof  # noqa: E402
    import decode_core  # noqa: E402
    import graph as ref_graph  # noqa: E402
    fk._module = _CpuExtension(fk)
    return SimpleNamespace(fk=fk, mm=mm, drum=drum, proof=proof, decode_core=decode_core,
                           graph=ref_graph)


class _CpuExtension:
    """Stands in for the CUDA extension object; see the module docstring."""

    def __init__(self, fk):
        self.fk = fk

    @staticmethod
    def _pos_factor(order, mask_f, edge_weight, is_score, scale):
        eid = order.long()
        mk = mask_f.reshape(-1)
        if mk.numel() == 1:
            m = torch.full((eid.numel(),), 1.0 if bool(mk[0]) else 0.0)
        else:
            m = (mk[eid] != 0).float()
        if edge_weight is not None and edge_weight.numel() > 0:
            ew = edge_weight.reshape(-1)[eid].float()
            m = m * (ew if is_score else torch.sigmoid(ew * float(scale)))
        return m

    def _expand(self, sp_b, sp_l, sp_e, sp_v, w, rgp, gr, gs, gc, col, order, m_pos, off, cap):
        fk = self.fk
        b, l, e, v, entry, rel, m = fk._expand_sparse3d_direction_cpu(
            sp_b, sp_l, sp_e, sp_v, w, rgp, gr, gs, gc, col, m_pos, off, cap)
        pos_ids = torch.arange(col.numel(), dtype=torch.int32)
        _, _, pos, _, _, _, _ = fk._expand_sparse3d_direction_cpu(
            sp_b, sp_l, sp_e, sp_v, w, rgp, gr, gs, gc, pos_ids, m_pos, off, cap)
        edge = order.long()[pos]
        nnz = sp_b.numel()
        offsets = torch.zeros(nnz + 1, dtype=torch.long)
        if entry.numel():
            offsets[1:] = torch.bincount(entry, minlength=nnz).cumsum(0)
        return b, l, e, v, entry, rel.to(torch.int16), m, offsets, edge

    def fastlog_forward_sparse3d_topk_cuda(self, sp_b, sp_l, sp_e, sp_v, w,
                                           oci, oo, orgp, ogr, ogs, ogc,
                                           ici, io, irgp, igr, igs, igc,
                                           mask_f, edge_weight, B, L, E, r_size, wot_i,
                                           topk_edges, is_score, scale):
        sp_v = sp_v.float()
        w = w.float()
        n = w.shape[2]
        o = self._expand(sp_b, sp_l, sp_e, sp_v, w, orgp, ogr, ogs, ogc, oci, oo,
                         self._pos_factor(oo, mask_f, edge_weight, is_score, scale), 0, topk_edges)
        i = self._expand(sp_b, sp_l, sp_e, sp_v, w, irgp, igr, igs, igc, ici, io,
                         self._pos_factor(io, mask_f, edge_weight, is_score, scale), r_size, topk_edges)
        if wot_i:
            ind_v = torch.zeros_like(sp_v)
        else:
            ind_v = sp_v * w[sp_b, sp_l, n - 1]
        return (o[0], o[1], o[2], o[3], i[0], i[1], i[2], i[3],
                sp_b.clone(), sp_l.clone(), sp_e.clone(), ind_v,
                o[4], o[5], o[6], i[4], i[5], i[6], o[7], i[7], o[8], i[8])

    def fastlog_backward_sparse3d_topk_cuda(self, gov, gob, gol, goe, giv, gib, gil, gie,
                                            gindv, gindb, gindl, ginde,
                                            sp_b, sp_l, sp_e, sp_v, w,
                                            ob, ol, oe, o_entry, o_rel, o_mask, o_off,
                                            ib, il, ie, i_entry, i_rel, i_mask, i_off,
                                            B, L, E, r_size, wot_i):
        fk = self.fk
        shape = [B, L, E]
        sp = lambda v, b, l, e: torch.sparse_coo_tensor(torch.stack([b, l, e]), v, shape).coalesce()
        ctx = SimpleNamespace(
            saved_tensors=(sp_b, sp_l, sp_e, sp_v.float(), w.float(),
                           ob, ol, oe, o_entry.long(), o_rel.long(), o_mask,
                           ib, il, ie, i_entry.long(), i_rel.long(), i_mask),
            B=B, L=L, E=E, r_size=r_size, wot_i=wot_i)
        res = fk.FastLogFunctionSparse3DCPU.backward(
            ctx, sp(gov, gob, gol, goe), sp(giv, gib, gil, gie), sp(gindv, gindb, gindl, ginde))
        return res[3], res[4]

    def fastlog_backward_sparse3d_topk_aligned_cuda(self, g_ori, o_entry, o_rel, o_mask,
                                                    g_inv, i_entry, i_rel, i_mask,
                                                    gindv, gindb, gindl, ginde,
                                                    sp_b, sp_l, sp_e, sp_v, w,
                                                    B, L, E, r_size, wot_i):
        fk = self.fk
        sp_v = sp_v.float()
        w = w.float()
        n = w.shape[2]
        grad_sp = torch.zeros_like(sp_v)
        grad_w = torch.zeros_like(w)
        for g, entry, rel, m, off in ((g_ori, o_entry, o_rel, o_mask, 0),
                                      (g_inv, i_entry, i_rel, i_mask, r_size)):
            if g.numel() == 0:
                continue
            nz = g != 0
            ent = entry.long()[nz]
            ch = rel.long()[nz] + off
            gm = g[nz] * m[nz]
            bb, ll = sp_b[ent], sp_l[ent]
            grad_sp.index_add_(0, ent, gm * w[bb, ll, ch])
            grad_w.view(-1).index_add_(0, (bb * L + ll) * n + ch, gm * sp_v[ent])
        if not wot_i and gindb.numel() > 0:
            gi = torch.sparse_coo_tensor(torch.stack([gindb, gindl, ginde]), gindv, [B, L, E]).coalesce()
            g = fk._gather_sparse3d_grad_at_entities(gi, sp_b, sp_l, sp_e, L, E)
            grad_sp += g * w[sp_b, sp_l, n - 1]
            grad_w.view(-1).index_add_(0, (sp_b * L + sp_l) * n + (n - 1), g * sp_v)
        return grad_sp, grad_w


def csr_tensors(ref, head, rel, tail, E):
    return ref.fk.build_csr_structure(torch.from_numpy(head.astype(np.int64)),
                                      torch.from_numpy(tail.astype(np.int64)),
                                      torch.from_numpy(rel.astype(np.int64)), E)


def coo_np(sp, prefix, out):
    sp = sp.coalesce()
    idx = sp.indices().numpy().astype(np.int64)
    out[prefix + "_idx"] = idx
    out[prefix + "_val"] = sp.values().detach().numpy().astype(np.float32)


def random_frontier(rng, B, L, E, per_row):
    keys = set()
    b_all, l_all, e_all = [], [], []
    for b in range(B):
        for l in range(L):
            ents = rng.choice(E, size=per_row, replace=False)
            for e in ents:
                b_all.append(b); l_all.append(l); e_all.append(int(e))
    b = np.array(b_all, np.int64); l = np.array(l_all, np.int64); e = np.array(e_all, np.int64)
    order = np.lexsort((e, l, b))
    vals = rng.uniform(0.05, 1.0, size=b.shape[0]).astype(np.float32)
    # a few exact value ties so argmax / max tie rules are exercised
    vals[::7] = np.float32(0.5)
    return b[order], l[order], e[order], vals


def op_case(ref, out, tag, kg, w, frontier, scores, mask, cap, agg, is_score, scale, rng):
    fk = ref.fk
    B, L, _ = w.shape
    E = kg.num_entities
    R = kg.num_relations
    csr = csr_tensors(ref, kg.head, kg.rel, kg.tail, E)
    sb, sl, se, sv = (torch.from_numpy(x) for x in frontier)
    sv = sv.clone().requires_grad_(True)
    wt = torch.from_numpy(w).clone().requires_grad_(True)
    ew = torch.from_numpy(scores if is_score else np.log(scores / (1 - scores + 1e-6)).astype(np.float32))
    ew = ew.clone().requires_grad_(True)
    mk = torch.from_numpy(mask.astype(np.float32))
    o, i, d = fk.FastLogFunctionSparse3DTopK.apply(
        sb, sl, se, sv, wt, *csr, mk, ew, B, L, E, R, False, int(cap), int(agg), bool(is_score), float(scale))
    coo_np(o, tag + "_ori", out)
    coo_np(i, tag + "_inv", out)
    coo_np(d, tag + "_ind", out)
    # seed gradients on each output's keys
    gs = []
    for name, t in (("ori", o), ("inv", i), ("ind", d)):
        t = t.coalesce()
        g = torch.from_numpy(rng.standard_normal(t._nnz()).astype(np.float32))
        out[f"{tag}_seed_{name}"] = g.numpy()
        gs.append((t.values() * g).sum())
    sum(gs).backward()
    out[tag + "_grad_sp"] = sv.grad.numpy()
    out[tag + "_grad_w"] = wt.grad.numpy()
    out[tag + "_grad_edge"] = ew.grad.numpy()
    out[tag + "_ew"] = ew.detach().numpy()
    if agg == 1:
        # the argmax message of every ori / inv output key, as (fact id, frontier entry)
        res = fk._module.fastlog_forward_sparse3d_topk_cuda(
            sb, sl, se, sv.detach(), wt.detach(), csr[1].int(), csr[3].int(), *csr[8:12],
            csr[5].int(), csr[7].int(), *csr[12:16], mk, ew.detach(), B, L, E, R, False, int(cap),
            bool(is_score), float(scale))
        for name, base, eb in (("ori", 0, 12), ("inv", 4, 15)):
            _, keys, _, raw_arg = fk._coalesce_sparse3d_max_with_arg(
                res[base], res[base + 1], res[base + 2], res[base + 3], B, L, E,
                tie_break=res[20 if name == "ori" else 21])
            edge = res[20 if name == "ori" else 21]
            entry = res[eb]
            out[f"{tag}_{name}_arg_edge"] = edge[raw_arg].numpy()
            out[f"{tag}_{name}_arg_entry"] = entry[raw_arg].numpy()
            out[f"{tag}_{name}_nmsg"] = np.array([res[base].numel()])


def fake_model(kg, logits, scores, tau=1.0):
    B, K, L, n = logits.shape
    logit_param = torch.from_numpy(logits).clone().requires_grad_(True)
    weight = torch.from_numpy(scores).clone().requires_grad_(True)
    model = SimpleNamespace(
        rules=L, entity_count=kg.num_entities, relation_count=kg.num_relations, step=K,
        tau_1=tau, edge_weight_mask=None, weight_override=None, weight_transform=None,
        gate_scope="all", supply_temperature=1.0, weight=weight, weight_param=weight,
        dropout=lambda x: x)
    model.build_rule_logits = lambda rels: logit_param
    return model, logit_param, weight


def proof_case(ref, out, tag, kg, heads, logits, scores, cap, topk_nodes, rng):
    facts = torch.from_numpy(np.stack([kg.head, kg.rel, kg.tail], 1).astype(np.int32))
    g = ref.graph.Graph(facts)
    model, lp, wt = fake_model(kg, logits, scores)
    args = SimpleNamespace(kernel_topk_edges=int(cap), kernel_topk_nodes=int(topk_nodes))
    hd = torch.from_numpy(heads)
    raw = ref.proof.kernel_sparse_scores(model, hd, torch.zeros_like(hd), g, args, is_training=True)
    raw = raw.coalesce()
    coo_np(raw, tag + "_final", out)
    seed = torch.from_numpy(rng.standard_normal(raw._nnz()).astype(np.float32))
    out[tag + "_seed"] = seed.numpy()
    (raw.values() * seed).sum().backward()
    out[tag + "_grad_logits"] = lp.grad.numpy()
    out[tag + "_grad_edge"] = wt.grad.numpy()


def max_decode_case(ref, out, tag, kg, heads, logits, scores, cap, topk):
    """The max-aggregation loop of src/model_mmDRUM_kernel_sp.py:388-445, then decode."""
    fk, mm = ref.fk, ref.mm
    E, R = kg.num_entities, kg.num_relations
    B, K, L, n = logits.shape
    csr = csr_tensors(ref, kg.head, kg.rel, kg.tail, E)
    mk = torch.ones(kg.num_triples)
    ew = torch.from_numpy(scores)
    sb = torch.arange(B).repeat_interleave(L)
    sl = torch.arange(L).repeat(B)
    se = torch.from_numpy(heads).repeat_interleave(L)
    state = torch.sparse_coo_tensor(torch.stack([sb, sl, se]), torch.ones(B * L), [B, L, E]).coalesce()
    final = None
    lg = torch.from_numpy(logits)
    for t in range(K):
        w_t = torch.softmax(lg[:, t], dim=-1)
        o, i, d = fk.FastLogFunctionSparse3DTopK.apply(
            state.indices()[0], state.indices()[1], state.indices()[2], state.values(), w_t,
            *csr, mk, ew, B, L, E, R, False, int(cap), 1, True, 1.0)
        s = mm.sparse3d_max(d, o, i)
        coo_np(s, f"{tag}_hop{t}_max", out)
        if t < K - 1:
            state = mm.norm_sp_3d(s)
        else:
            final = mm.norm_sp_3d_max(s)
    coo_np(final, tag + "_final", out)
    bounded = ref.proof.bound_sparse_scores(final)
    rows = ref.proof.sparse_candidate_rows(bounded)
    tails = np.full((B, topk), -1, np.int64)
    sc = np.zeros((B, topk), np.float32)
    for r, (tt, ss) in rows.items():
        ot, os_ = ref.decode_core.ordered_tail_scores(tt, ss, topk)
        tails[r, :len(ot)] = ot
        sc[r, :len(os_)] = os_
    out[tag + "_tails"] = tails
    out[tag + "_scores"] = sc


def reducer_case(ref, out, rng):
    """Bridge / model reducers with deliberate value ties."""
    mm, drum = ref.mm, ref.drum
    import src.fastlog_bridge as bridge  # noqa: E402
    B, L, E = 4, 3, 50
    states = []
    for s in range(3):
        nnz = 120
        b = rng.integers(0, B, nnz); l = rng.integers(0, L, nnz); e = rng.integers(0, E, nnz)
        v = rng.choice(np.array([0.0, 0.25, 0.5, 0.5, 1.0, 0.125, 0.75], np.float32), nnz)
        v = v + (rng.random(nnz) < 0.3) * rng.random(nnz).astype(np.float32)
        t = torch.sparse_coo_tensor(torch.from_numpy(np.stack([b, l, e])),
                                    torch.from_numpy(v.astype(np.float32)), [B, L, E]).coalesce()
        states.append(t)
        coo_np(t, f"red_in{s}", out)
    coo_np(bridge.sum_sparse3d_concat(*states), "red_concat", out)
    coo_np(bridge.sum_sp_3d(states[0]), "red_sum_sp_3d", out)
    coo_np(mm.max_sp_3d(states[0]), "red_max_sp_3d", out)
    coo_np(mm.sparse3d_max(*states), "red_sparse3d_max", out)
    coo_np(drum.normalize_sparse3d(states[1], 0.0, "mass"), "red_normalize_mass", out)
    coo_np(drum.normalize_sparse3d(states[1], 0.0, "none"), "red_normalize_none", out)
    coo_np(mm.norm_sp_3d(states[2]), "red_norm_sp_3d", out)
    coo_np(mm.norm_sp_3d_max(states[2]), "red_norm_sp_3d_max", out)
    # prune with distinct entity scores (torch.topk tie order is unspecified)
    v = torch.from_numpy(rng.uniform(0.1, 1.0, 200).astype(np.float32))
    b = torch.from_numpy(rng.integers(0, B, 200)); l = torch.from_numpy(rng.integers(0, L, 200))
    e = torch.from_numpy(rng.integers(0, E, 200))
    t = torch.sparse_coo_tensor(torch.stack([b, l, e]), v, [B, L, E]).coalesce()
    coo_np(t, "red_prune_in", out)
    coo_np(drum.prune_sparse3d_active_entities(t, 20), "red_prune20", out)
    # decode ordering with tied scores
    tails = rng.permutation(200)[:60]
    scores = rng.choice(np.array([0.9, 0.5, 0.5, 0.25, 0.1], np.float32), 60)
    ot, os_ = ref.decode_core.ordered_tail_scores(tails, scores, 25)
    out["ord_tails_in"] = tails.astype(np.int64); out["ord_scores_in"] = scores
    out["ord_tails"] = ot; out["ord_scores"] = os_


def prune_case(ref, out, kg, rng):
    """First-hop query pruning (decode_core.py:287-348) with a per-relation fake rule model."""
    R, E = kg.num_relations, kg.num_entities
    n = 2 * R + 1
    K, L = 2, 3
    logits = (rng.standard_normal((R, K, L, n)) * 2.5).astype(np.float32)
    logits[3] = 0.0                      # flat weights: no channel reaches the threshold
    logits[4] = 0.0
    logits[4, 0, :, 2 * R] = 20.0        # only the identity channel is active
    model = SimpleNamespace(relation_count=R, tau_1=0.8, emb=torch.zeros(1))
    model.build_rule_logits = lambda rels: torch.from_numpy(logits[int(rels[0])][None])
    facts = np.stack([kg.head, kg.rel, kg.tail], 1).astype(np.int64)
    supply = rng.random(kg.num_triples) < 0.8
    relations = [0, 1, 3, 4, 5, R - 1]
    args = SimpleNamespace(decode_query_prune="rule_first_hop", decode_query_rule_threshold=0.2)
    ref.decode_core.prepare_rule_first_hop_prune(model, relations, facts, supply, args)
    act, act_off, qs, q_off, kept, kept_off = [], [0], [], [0], [], [0]
    for r in relations:
        a = list(args._decode_query_active_channels[r])
        q = rng.integers(0, E, 300).astype(np.int64)
        k = ref.decode_core.rule_first_hop_query_heads(r, q.tolist(), args)
        act += a; act_off.append(len(act))
        qs.append(q); q_off.append(q_off[-1] + q.size)
        kept += k; kept_off.append(len(kept))
    cache = args._decode_query_channel_heads
    keys = sorted(cache)
    out.update(pf_logits=logits, pf_tau=np.array([0.8], np.float32), pf_threshold=np.array([0.2], np.float32),
               pf_head=kg.head, pf_rel=kg.rel, pf_tail=kg.tail, pf_E=np.array([E]), pf_R=np.array([R]),
               pf_supply=supply, pf_relations=np.array(relations, np.int64),
               pf_active=np.array(act, np.int64), pf_active_off=np.array(act_off, np.int64),
               pf_queries=np.concatenate(qs), pf_queries_off=np.array(q_off, np.int64),
               pf_kept=np.array(kept, np.int64), pf_kept_off=np.array(kept_off, np.int64),
               pf_cache_keys=np.array(keys, np.int64),
               pf_cache=np.concatenate([cache[c] for c in keys]) if keys else np.zeros(0, np.int64),
               pf_cache_off=np.cumsum([0] + [cache[c].size for c in keys]).astype(np.int64))


def accum_case(ref, out, rng):
    """The decode accumulator's best-k selection (decode.py:45-116) on synthetic rows:
    ordered candidate tails, per-query true and base (supplied) tail sets, empty cases and a
    repeated tail included."""
    import decode as ref_decode  # the reference's decode module (imports resolved via sys.path)
    acc = ref_decode._OracleRelationAccumulator()
    rows_t, rows_true, rows_base, best = [], [], [], []
    for q in range(60):
        n = int(rng.integers(0, 40)) if q % 7 else 0
        tails = rng.permutation(200)[:n].astype(np.int64)
        if q % 11 == 3 and n > 2:
            tails[-1] = tails[0]  # a repeated tail
        hits = tails[: min(n, 12)][rng.random(min(n, 12)) < 0.6]  # early candidates are often true
        true = np.unique(np.concatenate([hits, rng.choice(200, int(rng.integers(0, 25)), replace=False)])) \
            .astype(np.int64) if q % 5 else np.zeros(0, np.int64)
        base = rng.choice(200, int(rng.integers(0, 15)), replace=False).astype(np.int64)
        if q % 9 == 2:
            base = np.concatenate([base, base[:2]])  # duplicated base ids
        best.append(acc.add_row(tails, true, base))
        rows_t.append(tails); rows_true.append(true); rows_base.append(base)
    off = lambda rows: np.cumsum([0] + [r.size for r in rows]).astype(np.int64)  # noqa: E731
    out.update(ac_tails=np.concatenate(rows_t), ac_tails_off=off(rows_t),
               ac_true=np.concatenate(rows_true), ac_true_off=off(rows_true),
               ac_base=np.concatenate(rows_base), ac_base_off=off(rows_base),
               ac_best=np.array(best, np.int64),
               ac_counters=np.array([acc.candidate_total, acc.max_candidate_count, acc.query_count, acc.selected,
                                     acc.selected_wrong, acc.new, acc.new_true], np.int64))


def rules_case(ref, out, tag, R, H, K, L, B, tau, scale, seed, penalty=0.0, invert=False, table=None):
    """The rule-weight producer: SupplyGatedDRUM.build_rule_logits (drum.py:440-467) and the
    per-hop softmax of proof.py:571, forward and backward (loss = sum(w * G))."""
    torch.manual_seed(seed)
    rng = np.random.default_rng(seed)
    n = 2 * R + 1
    model = ref.drum.SupplyGatedDRUM(
        relation_channels=n, step=K, rules=L, entity_count=10, fact_count=4, emb_size=H, tau_1=tau, dropout=0.0,
        top_k_entities=8, top_k_mask=8, use_topk=True, supply_temperature=0.2, hard_threshold=0.5,
        rule_logit_init_scale=scale, rule_parametrization="target_table" if table is not None else "shared",
        norm_epsilon=0.0, norm_availability="mass", same_relation_channel_penalty=penalty, model_base="drum",
        target_table_relations=table)
    if invert:
        model._tclm_invert_rules = True
    rels = rng.integers(0, R, B).astype(np.int64)
    rels[: min(B, 3)] = rels[0]  # repeated relations
    rels_t = torch.from_numpy(rels)
    logits = model.build_rule_logits(rels_t)
    w = torch.stack([torch.softmax(logits[:, h] / model.tau_1, dim=-1) for h in range(K)])
    G = torch.from_numpy(rng.standard_normal(tuple(w.shape)).astype(np.float32))
    (w * G).sum().backward()
    pre = f"rl_{tag}_"
    out[pre + "dims"] = np.array([R, H, K, L, B], np.int64)
    out[pre + "tau"] = np.array([tau], np.float32)
    out[pre + "penalty"] = np.array([penalty], np.float32)
    out[pre + "invert"] = np.array([int(invert)], np.int64)
    out[pre + "rels"] = rels
    out[pre + "logits"] = logits.detach().numpy()
    out[pre + "w"] = w.detach().numpy()
    out[pre + "G"] = G.numpy()
    for name, prm in model.named_parameters():
        if name == "weight_param":
            continue
        key = name.replace(".", "__")
        out[pre + "p_" + key] = prm.detach().numpy()
        out[pre + "g_" + key] = (prm.grad if prm.grad is not None else torch.zeros_like(prm)).numpy()
    if table is not None:
        out[pre + "table_index"] = model.target_table_index.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository (majh3/miniKG_dev)")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", choices=("all", "prune", "accum", "rules"), default="all")
    a = ap.parse_args()
    torch.set_num_threads(1)  # index_put_/scatter_add_ are then sequential in index order
    ref = import_reference(a.ref)
    if a.only in ("all", "accum"):
        ac = {}
        accum_case(ref, ac, np.random.default_rng(8))
        np.savez_compressed(os.path.join(a.out, "golden_accum.npz"), **ac)
        print("wrote accum", len(ac))
        if a.only == "accum":
            return
    if a.only in ("all", "rules"):
        rl = {}
        rules_case(ref, rl, "a", R=9, H=48, K=3, L=2, B=12, tau=1.0, scale=1.0, seed=21)
        rules_case(ref, rl, "b", R=51, H=64, K=2, L=2, B=40, tau=0.7, scale=0.01, seed=22)
        rules_case(ref, rl, "c", R=6, H=16, K=3, L=2, B=7, tau=1.0, scale=1.0, seed=23, penalty=0.5, invert=True)
        rules_case(ref, rl, "d", R=6, H=16, K=2, L=2, B=9, tau=1.0, scale=1.0, seed=24, table=[1, 2, 4])
        np.savez_compressed(os.path.join(a.out, "golden_rules.npz"), **rl)
        print("wrote rules", len(rl))
        if a.only == "rules":
            return
    if a.only in ("all", "prune"):
        kg = sample_graph(900, 9, 9000, (("rel", ("zipf", 1.0)), ("head", (0.9, 2.0)), ("tail", (0.9, 2.0)),
                                         ("hubs", (0.05, 0.4))), seed=12, name="g2")
        pf = {}
        prune_case(ref, pf, kg, np.random.default_rng(7))
        np.savez_compressed(os.path.join(a.out, "golden_prune.npz"), **pf)
        print("wrote prune", len(pf))
        if a.only == "prune":
            return
    rng = np.random.default_rng(0)

    graphs = {
        "g1": sample_graph(600, 6, 5000, (("rel", ("zipf", 1.1)), ("head", (1.5, 6.0)), ("tail", (0.6, 1.0))),
                           seed=11, name="g1"),
        "g2": sample_graph(900, 9, 9000, (("rel", ("zipf", 1.0)), ("head", (0.9, 2.0)), ("tail", (0.9, 2.0)),
                                          ("hubs", (0.05, 0.4))), seed=12, name="g2"),
    }
    for gname, kg in graphs.items():
        out = {"head": kg.head, "rel": kg.rel, "tail": kg.tail,
               "E": np.array([kg.num_entities]), "R": np.array([kg.num_relations])}
        csr = csr_tensors(ref, kg.head, kg.rel, kg.tail, kg.num_entities)
        for k, t in enumerate(csr):
            out[f"csr{k}"] = t.numpy()
        n = 2 * kg.num_relations + 1
        B, L = 3, 2
        w = softmax_f32(rng.standard_normal((B, L, n)).astype(np.float32))
        frontier = random_frontier(rng, B, L, kg.num_entities, per_row=25)
        scores = rng.uniform(0.05, 1.0, kg.num_triples).astype(np.float32)
        scores[::5] = np.float32(0.5)  # exact ties between messages
        mask = np.ones(kg.num_triples, bool)
        out.update(op_w=w, op_b=frontier[0], op_l=frontier[1], op_e=frontier[2], op_v=frontier[3],
                   op_scores=scores)
        cases = [("sum_unc", UNCAPPED, 0, True), ("sum_cap", 7, 0, True), ("max_unc", UNCAPPED, 1, True),
                 ("max_cap", 7, 1, True), ("sum_logit", UNCAPPED, 0, False), ("sum_cap0", 0, 0, True)]
        for tag, cap, agg, is_score in cases:
            op_case(ref, out, tag, kg, w, frontier, scores, mask, cap, agg, is_score, 1.0, rng)
        # hop loop + backward, and the max decode
        Bq, K, Lq = 6, 3, 3
        heads = rng.integers(0, kg.num_entities, Bq).astype(np.int64)
        logits = rng.standard_normal((Bq, K, Lq, n)).astype(np.float32)
        pscores = rng.uniform(0.05, 1.0, kg.num_triples).astype(np.float32)
        out.update(pr_heads=heads, pr_logits=logits, pr_scores=pscores)
        proof_case(ref, out, "pr_unc", kg, heads, logits, pscores, UNCAPPED, 0, rng)
        proof_case(ref, out, "pr_cap", kg, heads, logits, pscores, 9, 0, rng)
        proof_case(ref, out, "pr_prune", kg, heads, logits, pscores, UNCAPPED, 40, rng)
        max_decode_case(ref, out, "dec_unc", kg, heads, logits, pscores, UNCAPPED, 10)
        max_decode_case(ref, out, "dec_cap", kg, heads, logits, pscores, 9, 10)
        np.savez_compressed(os.path.join(a.out, f"golden_{gname}.npz"), **out)
        print("wrote", gname, len(out), "arrays")
    red = {}
    reducer_case(ref, red, rng)
    np.savez_compressed(os.path.join(a.out, "golden_reducers.npz"), **red)
    print("wrote reducers", len(red))


if __name__ == "__main__":
    main()
