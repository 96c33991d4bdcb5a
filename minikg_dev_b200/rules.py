"""Rule-weight producer on the device: ``SupplyGatedDRUM.build_rule_logits`` (drum.py:440-467)
and the per-hop softmax of the hop loop (proof.py:569-571).

The reference builds, for every query row, the sequence ``[emb[rel]] * K + [emb[n - 1]]``
(drum.py:429-438), runs one bidirectional LSTM per rule over it and maps the first K outputs
through ``linear`` (2H -> n); the hop loop then takes ``softmax(rule_logits[:, hop] / tau_1)``.
Everything depends on the query only through its target relation, so here:

* ``RuleLogits`` runs the LSTMs and the linear layer once per distinct relation
  (``mkg_rule_logits_forward``: one block per (relation, rule, direction)), backward by
  ``mkg_rule_logits_backward`` (BPTT and weight gradients, fixed-order sums);
* the parametrisation variants of ``build_rule_logits`` (target table, same-relation channel
  penalty, TCLM inversion) are applied to those per-relation logits with the reference's own
  indexing (a few small torch ops);
* ``RuleSoftmax`` gathers each query's row and takes the softmax per hop
  (``mkg_rule_softmax_forward``: [K, B, L, n], the layout the hop loop consumes), backward
  summed over each relation's queries in a fixed order (``mkg_rule_softmax_backward``).

Kernels flag an out-of-range relation in the device error word (raised by the next checked
call, ``_native.raise_device_errors``); the product path has no CPU implementation.
"""
from __future__ import annotations

import torch

from . import _native as N


def _params(n: int, H: int, L: int, K: int, U: int, B: int = 1, tau: float = 1.0) -> N.RuleParams:
    return N.RuleParams(int(n), int(H), int(L), int(K), int(U), int(B), float(tau), 0)


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


def group_queries(rels: torch.Tensor):
    """(rel_u [U] sorted distinct relations, query_u [B] each query's row, query_ptr [U + 1],
    query_perm [B]): the queries of relation u are query_perm[query_ptr[u]:query_ptr[u + 1]]."""
    r = rels.reshape(-1).long()
    rel_u, query_u, counts = torch.unique(r, sorted=True, return_inverse=True, return_counts=True)
    qptr = torch.zeros(rel_u.numel() + 1, dtype=torch.int64, device=r.device)
    torch.cumsum(counts, 0, out=qptr[1:])
    qperm = torch.sort(query_u, stable=True).indices
    return rel_u.contiguous(), query_u.contiguous(), qptr, qperm.contiguous()


class RuleLogits(torch.autograd.Function):
    """logits_u [U, K, L, n] = the shared rule logits (drum.py:429-438) of relations rel_u."""

    @staticmethod
    def forward(ctx, emb, w_ih, w_hh, bias, w_lin, b_lin, rel_u, K: int):
        for t, what in ((emb, "emb"), (w_ih, "w_ih"), (w_hh, "w_hh"), (bias, "bias"), (w_lin, "w_lin"),
                        (b_lin, "b_lin"), (rel_u, "rel_u")):
            N.require_cuda(t, what)
        dev = emb.device
        n, H = int(emb.shape[0]), int(emb.shape[1])
        L = int(w_ih.shape[0])
        U = int(rel_u.numel())
        if tuple(w_ih.shape) != (L, 2, 4 * H, H) or tuple(w_hh.shape) != (L, 2, 4 * H, H) \
                or tuple(bias.shape) != (L, 2, 4 * H) or tuple(w_lin.shape) != (n, 2 * H) \
                or tuple(b_lin.shape) != (n,):
            raise RuntimeError("minikg_b200 rule producer: parameter shapes do not match emb [n, H]")
        p = _params(n, H, L, K, U)
        lib = N.load()
        emb_, w_ih_, w_hh_, bias_, w_lin_, b_lin_ = (_f32(t) for t in (emb, w_ih, w_hh, bias, w_lin, b_lin))
        rel = rel_u.long().contiguous()
        logits = torch.empty(U, K, L, n, dtype=torch.float32, device=dev)
        saved = N.workspace(lib.mkg_rule_saved_bytes(p), dev)
        N.check(lib.mkg_rule_logits_forward(p, emb_.data_ptr(), w_ih_.data_ptr(), w_hh_.data_ptr(), bias_.data_ptr(),
                                            w_lin_.data_ptr(), b_lin_.data_ptr(), rel.data_ptr(), logits.data_ptr(),
                                            saved.data_ptr(), saved.numel(), N.error_word(dev).data_ptr(),
                                            N.stream_handle(dev)), "rule_logits_forward")
        ctx.p, ctx.saved_buf = p, saved
        ctx.save_for_backward(emb_, w_ih_, w_hh_, w_lin_, rel)
        return logits

    @staticmethod
    def backward(ctx, grad_logits):
        emb, w_ih, w_hh, w_lin, rel = ctx.saved_tensors
        p, dev = ctx.p, emb.device
        lib = N.load()
        g = _f32(grad_logits)
        grad_emb = torch.empty_like(emb)
        grad_w_ih = torch.empty_like(w_ih)
        grad_w_hh = torch.empty_like(w_hh)
        grad_bias = torch.empty(w_ih.shape[:3], dtype=torch.float32, device=dev)
        grad_w_lin = torch.empty_like(w_lin)
        grad_b_lin = torch.empty(w_lin.shape[0], dtype=torch.float32, device=dev)
        ws = N.workspace(lib.mkg_rule_backward_workspace_bytes(p), dev)
        N.check(lib.mkg_rule_logits_backward(p, emb.data_ptr(), w_ih.data_ptr(), w_hh.data_ptr(), w_lin.data_ptr(),
                                             rel.data_ptr(), ctx.saved_buf.data_ptr(), ctx.saved_buf.numel(),
                                             g.data_ptr(), grad_emb.data_ptr(), grad_w_ih.data_ptr(),
                                             grad_w_hh.data_ptr(), grad_bias.data_ptr(), grad_w_lin.data_ptr(),
                                             grad_b_lin.data_ptr(), ws.data_ptr(), ws.numel(),
                                             N.error_word(dev).data_ptr(), N.stream_handle(dev)),
                "rule_logits_backward")
        return grad_emb, grad_w_ih, grad_w_hh, grad_bias, grad_w_lin, grad_b_lin, None, None


class RuleSoftmax(torch.autograd.Function):
    """w_hops [K, B, L, n] = softmax(logits_u[query_u[b], t, l, :] / tau) (proof.py:571)."""

    @staticmethod
    def forward(ctx, logits_u, query_u, qptr, qperm, tau: float):
        N.require_cuda(logits_u, "rule logits")
        dev = logits_u.device
        U, K, L, n = (int(s) for s in logits_u.shape)
        B = int(query_u.numel())
        p = _params(n, 1, L, K, U, B, tau)
        x = _f32(logits_u)
        qu = query_u.long().contiguous()
        w = torch.empty(K, B, L, n, dtype=torch.float32, device=dev)
        N.check(N.load().mkg_rule_softmax_forward(p, x.data_ptr(), qu.data_ptr(), w.data_ptr(),
                                                  N.error_word(dev).data_ptr(), N.stream_handle(dev)),
                "rule_softmax_forward")
        ctx.p = p
        ctx.save_for_backward(w, qptr.long().contiguous(), qperm.long().contiguous())
        return w

    @staticmethod
    def backward(ctx, grad_w):
        w, qptr, qperm = ctx.saved_tensors
        p, dev = ctx.p, w.device
        lib = N.load()
        g = _f32(grad_w)
        out = torch.empty(p.U, p.K, p.L, p.n, dtype=torch.float32, device=dev)
        ws = N.workspace(lib.mkg_rule_softmax_workspace_bytes(p), dev)
        N.check(lib.mkg_rule_softmax_backward(p, w.data_ptr(), g.data_ptr(), qptr.data_ptr(), qperm.data_ptr(),
                                              out.data_ptr(), ws.data_ptr(), ws.numel(),
                                              N.error_word(dev).data_ptr(), N.stream_handle(dev)),
                "rule_softmax_backward")
        return out, None, None, None, None


# ------------------------------------------------------------------ the model's producer
def lstm_params(model):
    """(w_ih, w_hh, bias) stacked from ``model.lstm`` (one ``nn.LSTM(H, H, 1, bidirectional=True)``
    per rule, drum.py:305): [L, 2, 4H, H], [L, 2, 4H, H], [L, 2, 4H] (b_ih + b_hh)."""
    w_ih, w_hh, bias = [], [], []
    for m in model.lstm:
        if m.num_layers != 1 or not m.bidirectional or m.input_size != m.hidden_size or m.proj_size:
            raise RuntimeError("minikg_b200 rule producer: expects single-layer bidirectional LSTMs of size H -> H")
        w_ih.append(torch.stack([m.weight_ih_l0, m.weight_ih_l0_reverse]))
        w_hh.append(torch.stack([m.weight_hh_l0, m.weight_hh_l0_reverse]))
        if m.bias:
            bias.append(torch.stack([m.bias_ih_l0 + m.bias_hh_l0, m.bias_ih_l0_reverse + m.bias_hh_l0_reverse]))
        else:
            bias.append(m.weight_ih_l0.new_zeros(2, m.weight_ih_l0.shape[0]))
    return torch.stack(w_ih), torch.stack(w_hh), torch.stack(bias)


def shared_rule_logits(model, rel_u: torch.Tensor) -> torch.Tensor:
    """``_shared_rule_logits`` (drum.py:429-438) for distinct relations: [U, K, L, n]."""
    w_ih, w_hh, bias = lstm_params(model)
    lin = model.linear
    b_lin = lin.bias if lin.bias is not None else lin.weight.new_zeros(lin.weight.shape[0])
    return RuleLogits.apply(model.emb, w_ih, w_hh, bias, lin.weight, b_lin, rel_u, int(model.step))


def _invert(logits: torch.Tensor, R: int) -> torch.Tensor:
    """tclm_invert_rule_logits (drum.py:238-243): swap the ori / inv channel blocks, reverse the hops."""
    return torch.flip(torch.cat([logits[..., R:2 * R], logits[..., :R], logits[..., 2 * R:]], dim=-1), dims=[1])


def relation_rule_logits(model, rel_u: torch.Tensor) -> torch.Tensor:
    """``build_rule_logits`` (drum.py:440-467) for distinct relations rel_u: [U, K, L, n]."""
    rel_u = rel_u.long()
    if getattr(model, "rule_parametrization", "shared") == "target_table":
        row = model.target_table_index[rel_u]
        mapped = row >= 0
        if bool(mapped.all().item()):
            logits = model.target_rule_logits[row]
        else:
            logits = shared_rule_logits(model, rel_u)
            if bool(mapped.any().item()):
                table = model.target_rule_logits[row.clamp_min(0)]
                logits = torch.where(mapped.view(-1, 1, 1, 1), table, logits)
    else:
        logits = shared_rule_logits(model, rel_u)
    R = int(model.relation_count)
    pen = float(getattr(model, "same_relation_channel_penalty", 0.0) or 0.0)
    if pen > 0:
        rows = torch.arange(rel_u.numel(), device=rel_u.device)
        logits = logits.clone()
        logits[rows, :, :, rel_u] -= pen
        logits[rows, :, :, rel_u + R] -= pen
    if getattr(model, "_tclm_invert_rules", False):
        logits = _invert(logits, R)
    elif getattr(model, "_tclm_selective_inverse", None) is not None:
        inv_mask = model._tclm_selective_inverse[rel_u].bool()
        if inv_mask.any():
            logits = torch.where(inv_mask.view(-1, 1, 1, 1), _invert(logits, R), logits)
    return logits


def has_lstm_producer(model) -> bool:
    """True for a model with SupplyGatedDRUM's producer attributes (drum.py:303-306)."""
    return all(hasattr(model, a) for a in ("emb", "lstm", "linear", "step", "relation_count"))


def build_rule_logits(model, target_rel: torch.Tensor) -> torch.Tensor:
    """Drop-in for ``SupplyGatedDRUM.build_rule_logits`` (drum.py:440-467): [B, K, L, n]."""
    rel_u, query_u, _, _ = group_queries(target_rel)
    return relation_rule_logits(model, rel_u).index_select(0, query_u)


def rule_weights(model, rels: torch.Tensor, tau: float | None = None) -> torch.Tensor:
    """w_hops [K, B, L, n] = softmax(build_rule_logits(rels)[:, hop] / tau_1) for every hop, the
    rule weights ``kernel_sparse_scores`` feeds the op (proof.py:524, 569-571)."""
    tau = float(model.tau_1 if tau is None else tau)
    if has_lstm_producer(model):
        rel_u, query_u, qptr, qperm = group_queries(rels)
        return RuleSoftmax.apply(relation_rule_logits(model, rel_u), query_u, qptr, qperm, tau)
    # a model with its own producer: its logits [B, K, L, n], one row per query
    return rule_weights_from_logits(model.build_rule_logits(rels), tau)


def rule_weights_from_logits(logits: torch.Tensor, tau: float) -> torch.Tensor:
    """softmax(logits[:, hop] / tau) for every hop of per-query logits [B, K, L, n] -> [K, B, L, n]."""
    B = int(logits.shape[0])
    ar = torch.arange(B, dtype=torch.int64, device=logits.device)
    qptr = torch.arange(B + 1, dtype=torch.int64, device=logits.device)
    return RuleSoftmax.apply(logits, ar, qptr, ar, float(tau))
