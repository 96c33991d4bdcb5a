"""The bridge reducers (``minikg_dev_b200.sparse_reducers``, csrc/mkg_reduce.cu) on the GPU.

Against the golden vectors the reference's own helpers produced (keys exact, maxima and the
ordered normalisations bit-exact, sums within fp32 rounding), against the oracle on larger
random states with duplicate keys and tied values (the tie rules: lowest rule for
``max_sp_3d``, earliest argument for ``sparse3d_max``, seen through where the gradient of
each maximum lands), and gradients against float64 dense autograd of the same reductions.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fastlog_oracle as O
from tests.conftest import load_golden

DEV = torch.device("cuda", 0)
B, L, E = 4, 3, 50


def _sp(keys, vals, shape, grad=False):
    """Sparse COO on the device from flat keys (row-major over ``shape``)."""
    keys = np.asarray(keys, np.int64)
    idx = []
    rest = keys
    for d in range(len(shape) - 1, 0, -1):
        idx.append(rest % shape[d])
        rest = rest // shape[d]
    idx.append(rest)
    v = torch.tensor(np.asarray(vals, np.float32), device=DEV, requires_grad=grad)
    return torch.sparse_coo_tensor(torch.tensor(np.stack(idx[::-1]), device=DEV), v, shape).coalesce(), v


def _np(s):
    s = s.coalesce()
    idx = s.indices().cpu().numpy()
    key = idx[0]
    for d in range(1, idx.shape[0]):
        key = key * s.shape[d] + idx[d]
    return key, s.values().detach().cpu().numpy()


def _golden(g, prefix):
    idx = g[prefix + "_idx"]
    key = idx[0]
    dims = (B, L, E) if idx.shape[0] == 3 else (B, E)
    for d in range(1, idx.shape[0]):
        key = key * dims[d] + idx[d]
    return key, g[prefix + "_val"]


@pytest.mark.gpu
def test_reducers_vs_golden():
    from minikg_dev_b200 import sparse_reducers as R
    g = load_golden("reducers")
    ins = [_golden(g, f"red_in{s}") for s in range(3)]
    st = [_sp(k, v, (B, L, E))[0] for k, v in ins]

    def check(prefix, got, exact):
        gk, gv = _golden(g, prefix)
        k, v = _np(got)
        np.testing.assert_array_equal(k, gk, err_msg=prefix)
        if exact:
            np.testing.assert_array_equal(v, gv, err_msg=prefix)
        else:
            np.testing.assert_allclose(v, gv, rtol=1e-6, atol=1e-7, err_msg=prefix)

    check("red_concat", R.sum_sparse3d_concat(*st), False)
    check("red_sum_sp_3d", R.sum_sp_3d(st[0]), False)
    check("red_max_sp_3d", R.max_sp_3d(st[0]), True)
    check("red_sparse3d_max", R.sparse3d_max(*st), True)
    check("red_normalize_mass", R.normalize_sparse3d(st[1], 0.0, "mass"), True)
    check("red_normalize_none", R.normalize_sparse3d(st[1], 0.0, "none"), True)
    check("red_norm_sp_3d", R.norm_sp_3d(st[2]), True)
    check("red_norm_sp_3d_max", R.norm_sp_3d_max(st[2]), True)
    pk, pv = _golden(g, "red_prune_in")
    check("red_prune20", R.prune_sparse3d_active_entities(_sp(pk, pv, (B, L, E))[0], 20), True)


def _random_states(seed, Bq=7, Lq=4, Eq=300, n=3, ties=True):
    rng = np.random.default_rng(seed)
    states = []
    for s in range(n):
        keys = np.unique(rng.integers(0, Bq * Lq * Eq, 900 + 50 * s))
        vals = rng.choice(np.array([0.25, 0.5, 0.75, 1.0], np.float32), keys.size) if ties else \
            rng.uniform(0.01, 1.0, keys.size).astype(np.float32)
        vals[rng.random(keys.size) < 0.03] = 0.0  # explicit zeros
        states.append((keys, vals))
    return states, (Bq, Lq, Eq)


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [0, 1])
def test_reducers_vs_oracle_with_ties(seed):
    from minikg_dev_b200 import sparse_reducers as R
    states, (Bq, Lq, Eq) = _random_states(seed)
    sp = [_sp(k, v, (Bq, Lq, Eq), grad=True) for k, v in states]
    # sums
    k, v = _np(R.sum_sparse3d_concat(*[s for s, _ in sp]))
    wk, wv = O.sum_sparse3d_concat(*states)
    np.testing.assert_array_equal(k, wk)
    np.testing.assert_allclose(v, wv, rtol=1e-6, atol=1e-7)
    k, v = _np(R.sum_sp_3d(sp[0][0]))
    wk, wv = O.sum_sp_3d(states[0], Lq, Eq)
    np.testing.assert_array_equal(k, wk)
    np.testing.assert_allclose(v, wv, rtol=1e-6, atol=1e-7)
    # max over rules: values exact, and each maximum's gradient lands on the lowest tied rule
    out = R.max_sp_3d(sp[0][0])
    k, v = _np(out)
    wk, wv = O.max_sp_3d(states[0], Lq, Eq)
    np.testing.assert_array_equal(k, wk)
    np.testing.assert_array_equal(v, wv)
    out.values().sum().backward()
    g = sp[0][1].grad.cpu().numpy()
    keys0, vals0 = states[0]
    b, l, e = O.split3(keys0, Lq, Eq)
    for kk in wk[:200]:
        bb, ee = kk // Eq, kk % Eq
        cand = np.nonzero((b == bb) & (e == ee))[0]
        best = cand[np.argmax(vals0[cand])]  # first maximum in (l) order
        assert g[best] == 1.0 and g[cand].sum() == 1.0
    # element-wise max across states: values exact, the earliest argument wins ties
    sp = [_sp(k, v, (Bq, Lq, Eq), grad=True) for k, v in states]
    out = R.sparse3d_max(*[s for s, _ in sp])
    k, v = _np(out)
    wk, wv, wslot = O.sparse3d_max(states, Lq, Eq)
    np.testing.assert_array_equal(k, wk)
    np.testing.assert_array_equal(v, wv)
    out.values().sum().backward()
    for j, kk in enumerate(wk[:300]):
        s_win = int(wslot[j])
        pos = np.searchsorted(states[s_win][0], kk)
        assert sp[s_win][1].grad[pos].item() == 1.0
    # normalisations: bit-exact against the oracle's in-order fp32 sums
    sp = [_sp(k, v, (Bq, Lq, Eq)) for k, v in states]
    for av in ("mass", "none"):
        k, v = _np(R.normalize_sparse3d(sp[1][0], 0.0, av))
        wk, wv = O.normalize_sparse3d(states[1], Bq, Lq, Eq, 0.0, av)
        np.testing.assert_array_equal(k, wk)
        np.testing.assert_array_equal(v, wv)
    k, v = _np(R.norm_sp_3d(sp[2][0]))
    wk, wv = O.norm_sp_3d(states[2], Bq, Lq, Eq)
    np.testing.assert_array_equal(k, wk)
    np.testing.assert_array_equal(v, wv)
    k, v = _np(R.prune_sparse3d_active_entities(sp[2][0], 40))
    wk, wv = O.prune_sparse3d_active_entities(states[2], Eq, 40)
    np.testing.assert_array_equal(k, wk)
    np.testing.assert_array_equal(v, wv)


@pytest.mark.gpu
def test_reducer_gradients_vs_dense_autograd():
    """d/dvalues of concat-sum -> normalize (mass) -> sum over rules, against the same chain
    on dense float64 tensors."""
    from minikg_dev_b200 import sparse_reducers as R
    states, (Bq, Lq, Eq) = _random_states(5, ties=False)
    sp = [_sp(k, v, (Bq, Lq, Eq), grad=True) for k, v in states]
    out = R.sum_sp_3d(R.normalize_sparse3d(R.sum_sparse3d_concat(*[s for s, _ in sp]), 0.0, "mass"))
    k, v = _np(out)
    seed = np.random.default_rng(9).standard_normal(k.size)
    (out.values() * torch.tensor(seed, device=DEV, dtype=torch.float32)).sum().backward()
    dense_in = []
    for keys, vals in states:
        d = torch.zeros(Bq * Lq * Eq, dtype=torch.float64)
        d[torch.from_numpy(keys)] = torch.from_numpy(vals.astype(np.float64))
        dense_in.append(d.requires_grad_(True))
    y = sum(dense_in).view(Bq, Lq, Eq)
    # the normalisation drops zero sums before its row sums: they get no gradient through d
    den = (y * (y != 0)).sum(dim=2, keepdim=True)
    den = torch.where(den == 0, torch.ones_like(den), den)  # empty rows: no NaN in the masked branch
    x = torch.where(y != 0, y / den * den.clamp_max(1.0), torch.zeros_like(y))
    z = x.sum(dim=1).reshape(-1)
    gz = torch.zeros_like(z)
    gz[torch.from_numpy(k)] = torch.from_numpy(seed)
    np.testing.assert_allclose(v, z.detach().numpy()[k], rtol=1e-5, atol=1e-6)
    (z * gz).sum().backward()
    for (keys, _), (_, vt), d in zip(states, sp, dense_in):
        np.testing.assert_allclose(vt.grad.cpu().numpy(), d.grad.numpy()[keys], rtol=1e-5, atol=1e-6)


def test_bridge_reducers_have_no_torch_sort_composition():
    """The bridge reducers reduce on the device kernel, not with torch's argsort /
    unique_consecutive / scatter_reduce."""
    src = (Path(__file__).resolve().parent.parent / "minikg_dev_b200" / "sparse_reducers.py").read_text()
    for word in ("argsort", "unique_consecutive", "scatter_reduce", "index_put_"):
        assert word not in src.split('"""', 2)[2], word
