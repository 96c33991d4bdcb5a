"""Rule-weight producer (drum.py:429-467 + proof.py:569-571): the oracle against golden vectors
from the reference's SupplyGatedDRUM (CPU), and the CUDA producer through the C ABI against the
golden vectors and the oracle (GPU)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fastlog_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_rules.npz"
CASES = ("a", "b", "c", "d")
# fp32 against the float64 oracle / the reference's fp32 CPU run; the absolute part scales
# with the tensor (logits and gradients of a 0.01-scaled initialisation are small)
FWD_TOL = dict(rtol=1e-5, scale=1e-6)
GRAD_TOL = dict(rtol=1e-4, scale=1e-5)   # backpropagation through K + 1 LSTM steps


def close(got, want, rtol, scale, err_msg=""):
    want = np.asarray(want, np.float64)
    atol = scale * max(float(np.abs(want).max(initial=0.0)), 1e-30)
    np.testing.assert_allclose(np.asarray(got, np.float64), want, rtol=rtol, atol=atol, err_msg=err_msg)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def case(g, tag):
    p = f"rl_{tag}_"
    R, H, K, L, B = (int(x) for x in g[p + "dims"])
    params = {"emb": g[p + "p_emb"], "w_lin": g[p + "p_linear__weight"], "b_lin": g[p + "p_linear__bias"], "lstm": []}
    grads = {"emb": g[p + "g_emb"], "w_lin": g[p + "g_linear__weight"], "b_lin": g[p + "g_linear__bias"],
             "lstm": []}
    for l in range(L):
        q = f"lstm__{l}__"
        prm, grd = {}, {}
        for key, name in (("w_ih", "weight_ih_l0"), ("w_hh", "weight_hh_l0"), ("b_ih", "bias_ih_l0"),
                          ("b_hh", "bias_hh_l0")):
            prm[key] = np.stack([g[p + "p_" + q + name], g[p + "p_" + q + name + "_reverse"]])
            grd[key] = np.stack([g[p + "g_" + q + name], g[p + "g_" + q + name + "_reverse"]])
        params["lstm"].append(prm)
        grads["lstm"].append(grd)
    table_index = g[p + "table_index"] if p + "table_index" in g.files else None
    table = g[p + "p_target_rule_logits"] if table_index is not None else None
    if table is not None:
        grads["table"] = g[p + "g_target_rule_logits"]
    return dict(R=R, H=H, K=K, L=L, B=B, tau=float(g[p + "tau"][0]), penalty=float(g[p + "penalty"][0]),
                invert=bool(g[p + "invert"][0]), rels=g[p + "rels"], params=params, grads=grads,
                table_index=table_index, table=table, logits=g[p + "logits"], w=g[p + "w"], G=g[p + "G"])


def check_grads(got, want, L, what):
    close(got["emb"], want["emb"], **GRAD_TOL, err_msg=f"{what} emb")
    close(got["w_lin"], want["w_lin"], **GRAD_TOL, err_msg=f"{what} w_lin")
    close(got["b_lin"], want["b_lin"], **GRAD_TOL, err_msg=f"{what} b_lin")
    if "table" in want:
        close(got["table"], want["table"], **GRAD_TOL, err_msg=f"{what} table")
    for l in range(L):
        gl, wl = got["lstm"][l], want["lstm"][l]
        for key in ("w_ih", "w_hh"):
            close(gl[key], wl[key], **GRAD_TOL, err_msg=f"{what} rule {l} {key}")
        close(gl["b"], wl["b_ih"], **GRAD_TOL, err_msg=f"{what} rule {l} b_ih")
        close(gl["b"], wl["b_hh"], **GRAD_TOL, err_msg=f"{what} rule {l} b_hh")


def oracle_run(c):
    logits, bwd = O.build_rule_logits(c["params"], c["rels"], c["K"], c["R"], c["penalty"], c["invert"],
                                      c["table_index"], c["table"])
    w = O.rule_softmax(logits, c["tau"])
    grads = bwd(O.rule_softmax_backward(w, c["G"].astype(np.float64), c["tau"]))
    return logits, w, grads


@pytest.mark.parametrize("tag", CASES)
def test_oracle_matches_golden(golden, tag):
    c = case(golden, tag)
    logits, w, grads = oracle_run(c)
    close(logits, c["logits"], **FWD_TOL)
    close(w, c["w"], **FWD_TOL)
    want = c["grads"]
    if "table" in want:
        close(grads["table"], want["table"], **GRAD_TOL)
    if "emb" not in grads:  # every relation had a table row: the shared producer did not run
        assert not np.any(want["emb"]) and not np.any(want["lstm"][0]["w_ih"])
        return
    check_grads(grads, want, c["L"], tag)


def test_oracle_invert_is_an_involution():
    x = np.random.default_rng(0).standard_normal((3, 4, 2, 13))
    np.testing.assert_array_equal(O.invert_rule_logits(O.invert_rule_logits(x, 6), 6), x)


# ------------------------------------------------------------------------------ GPU
class RuleModel(torch.nn.Module):
    """The producer attributes of SupplyGatedDRUM (drum.py:303-330) loaded with given values."""

    def __init__(self, c, device):
        super().__init__()
        p, H, L, R = c["params"], c["H"], c["L"], c["R"]
        n = 2 * R + 1
        self.relation_count, self.step, self.rules, self.tau_1 = R, c["K"], L, c["tau"]
        self.emb = torch.nn.Parameter(torch.tensor(p["emb"]))
        self.lstm = torch.nn.ModuleList(torch.nn.LSTM(H, H, 1, bidirectional=True) for _ in range(L))
        self.linear = torch.nn.Linear(2 * H, n)
        with torch.no_grad():
            for l, m in enumerate(self.lstm):
                lp = p["lstm"][l]
                for key, name in (("w_ih", "weight_ih_l0"), ("w_hh", "weight_hh_l0"), ("b_ih", "bias_ih_l0"),
                                  ("b_hh", "bias_hh_l0")):
                    getattr(m, name).copy_(torch.tensor(lp[key][0]))
                    getattr(m, name + "_reverse").copy_(torch.tensor(lp[key][1]))
            self.linear.weight.copy_(torch.tensor(p["w_lin"]))
            self.linear.bias.copy_(torch.tensor(p["b_lin"]))
        self.same_relation_channel_penalty = c["penalty"]
        self._tclm_invert_rules = c["invert"]
        if c["table_index"] is not None:
            self.rule_parametrization = "target_table"
            self.register_buffer("target_table_index", torch.tensor(c["table_index"]))
            self.target_rule_logits = torch.nn.Parameter(torch.tensor(c["table"]))
        else:
            self.rule_parametrization = "shared"
        self.to(device)

    def grads(self):
        out = {"emb": self.emb.grad, "w_lin": self.linear.weight.grad, "b_lin": self.linear.bias.grad, "lstm": []}
        for m in self.lstm:
            gl = {}
            for key, name in (("w_ih", "weight_ih_l0"), ("w_hh", "weight_hh_l0"), ("b_ih", "bias_ih_l0"),
                              ("b_hh", "bias_hh_l0")):
                a, b = getattr(m, name).grad, getattr(m, name + "_reverse").grad
                gl[key] = None if a is None else torch.stack([a, b])
            out["lstm"].append(gl)
        if self.rule_parametrization == "target_table":
            out["table"] = self.target_rule_logits.grad
        return out


def _np(t):
    return None if t is None else t.detach().double().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("tag", CASES)
def test_gpu_producer_matches_golden(golden, tag):
    from minikg_dev_b200 import rules
    c = case(golden, tag)
    dev = torch.device("cuda")
    model = RuleModel(c, dev)
    rels = torch.tensor(c["rels"], device=dev)
    logits = rules.build_rule_logits(model, rels)
    close(_np(logits), c["logits"], **FWD_TOL)
    w = rules.rule_weights(model, rels)
    close(_np(w), c["w"], **FWD_TOL)
    (w * torch.tensor(c["G"], device=dev)).sum().backward()
    from minikg_dev_b200 import _native as N
    N.raise_device_errors(dev)
    got = model.grads()
    want = c["grads"]
    if "table" in want:
        close(_np(got["table"]), want["table"], **GRAD_TOL)
    shared_ran = c["table_index"] is None or not (c["table_index"][c["rels"]] >= 0).all()
    if not shared_ran:
        assert got["emb"] is None and got["lstm"][0]["w_ih"] is None
        return
    close(_np(got["emb"]), want["emb"], **GRAD_TOL)
    close(_np(got["w_lin"]), want["w_lin"], **GRAD_TOL)
    close(_np(got["b_lin"]), want["b_lin"], **GRAD_TOL)
    for l in range(c["L"]):
        for key in ("w_ih", "w_hh", "b_ih", "b_hh"):
            close(_np(got["lstm"][l][key]), want["lstm"][l][key], **GRAD_TOL,
                                       err_msg=f"rule {l} {key}")


def synthetic_case(R, H, K, L, B, tau, scale, seed, distinct=None):
    rng = np.random.default_rng(seed)
    n = 2 * R + 1
    s = 1.0 / np.sqrt(H)
    params = {"emb": rng.uniform(-1, 1, (n, H)).astype(np.float32),
              "w_lin": (rng.uniform(-1, 1, (n, 2 * H)) * scale / np.sqrt(2 * H)).astype(np.float32),
              "b_lin": (rng.uniform(-1, 1, n) * scale / np.sqrt(2 * H)).astype(np.float32), "lstm": []}
    for _ in range(L):
        params["lstm"].append({k: rng.uniform(-s, s, shape).astype(np.float32) for k, shape in
                               (("w_ih", (2, 4 * H, H)), ("w_hh", (2, 4 * H, H)), ("b_ih", (2, 4 * H)),
                                ("b_hh", (2, 4 * H)))})
    pool = rng.choice(R, distinct, replace=False) if distinct else np.arange(R)
    rels = rng.choice(pool, B).astype(np.int64)
    return dict(R=R, H=H, K=K, L=L, B=B, tau=tau, penalty=0.0, invert=False, rels=rels, params=params,
                table_index=None, table=None, G=rng.standard_normal((K, B, L, n)).astype(np.float32))


SIZES = {
    # (R, H, K, L, B, tau, scale, distinct relations)
    "family_train": (12, 48, 3, 3, 512, 1.0, 1.0, None),
    "codex_train": (51, 64, 3, 3, 256, 1.0, 1.0, None),
    "wikidata_decode": (822, 64, 2, 4, 256, 1.0, 1.0, 1),
    "freebase_batch": (14824, 64, 2, 4, 128, 0.5, 1.0, 40),
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(SIZES))
def test_gpu_producer_matches_oracle(name):
    from minikg_dev_b200 import rules
    R, H, K, L, B, tau, scale, distinct = SIZES[name]
    c = synthetic_case(R, H, K, L, B, tau, scale, seed=len(name), distinct=distinct)
    dev = torch.device("cuda")
    model = RuleModel(c, dev)
    rels = torch.tensor(c["rels"], device=dev)
    w = rules.rule_weights(model, rels)
    logits, w_o, grads = oracle_run(c)
    close(_np(w), w_o, **FWD_TOL)
    close(_np(rules.build_rule_logits(model, rels)), logits, **FWD_TOL)
    (w * torch.tensor(c["G"], device=dev)).sum().backward()
    got = model.grads()
    for key in ("emb", "w_lin", "b_lin"):
        close(_np(got[key]), grads[key], **GRAD_TOL, err_msg=key)
    for l in range(L):
        for key, gk in (("w_ih", "w_ih"), ("w_hh", "w_hh"), ("b_ih", "b"), ("b_hh", "b")):
            close(_np(got["lstm"][l][key]), grads["lstm"][l][gk], **GRAD_TOL,
                                       err_msg=f"rule {l} {key}")


@pytest.mark.gpu
def test_gpu_producer_rejects_bad_relation():
    from minikg_dev_b200 import _native as N, rules
    c = synthetic_case(5, 16, 2, 2, 4, 1.0, 1.0, seed=3)
    dev = torch.device("cuda")
    model = RuleModel(c, dev)
    with pytest.raises(RuntimeError, match="rule producer"):
        rules.rule_weights(model, torch.tensor([0, 1, 11, 2], device=dev))
        N.raise_device_errors(dev)
    # the context stays usable
    w = rules.rule_weights(model, torch.tensor([0, 1, 3, 2], device=dev))
    N.raise_device_errors(dev)
    assert torch.isfinite(w).all()


@pytest.mark.gpu
def test_gpu_producer_deterministic():
    from minikg_dev_b200 import rules
    c = synthetic_case(51, 64, 3, 3, 256, 1.0, 1.0, seed=5)
    dev = torch.device("cuda")
    outs = []
    for _ in range(2):
        model = RuleModel(c, dev)
        w = rules.rule_weights(model, torch.tensor(c["rels"], device=dev))
        (w * torch.tensor(c["G"], device=dev)).sum().backward()
        outs.append([w.detach().clone(), model.emb.grad.clone(), model.lstm[0].weight_hh_l0.grad.clone(),
                     model.linear.weight.grad.clone()])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


# ------------------------------------------------------------------------------ host logic (CPU)
def test_group_queries_csr():
    """Distinct relations, each query's row and the per-relation query CSR (stable order)."""
    from minikg_dev_b200.rules import group_queries
    rels = torch.tensor([5, 2, 5, 9, 2, 2, 7, 5])
    rel_u, query_u, qptr, qperm = group_queries(rels)
    assert rel_u.tolist() == [2, 5, 7, 9]
    assert query_u.tolist() == [1, 0, 1, 3, 0, 0, 2, 1]
    assert qptr.tolist() == [0, 3, 6, 7, 8]
    assert qperm.tolist() == [1, 4, 5, 0, 2, 7, 6, 3]
    for u in range(rel_u.numel()):
        members = qperm[qptr[u]:qptr[u + 1]]
        assert (rels[members] == rel_u[u]).all()


def test_dense_cap_routing():
    """The fused loop takes caps 0..255 (a cap <= 0 takes no edge) and uncapped hops."""
    from minikg_dev_b200.proof import DENSE_CAP_MAX, UNCAPPED, dense_cap
    assert dense_cap(UNCAPPED) == UNCAPPED and dense_cap(1 << 62) == UNCAPPED
    assert dense_cap(100) == 100 and dense_cap(DENSE_CAP_MAX) == DENSE_CAP_MAX
    assert dense_cap(0) == 0 and dense_cap(-3) == 0
    assert dense_cap(DENSE_CAP_MAX + 1) is None and dense_cap(1000) is None
