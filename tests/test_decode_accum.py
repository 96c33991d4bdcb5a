"""The decode accumulator (best-k cut per candidate row) against the reference's own outputs."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import fastlog_oracle as O


@pytest.fixture(scope="module")
def ac():
    return load_golden("accum")


def _rows(z, name):
    off = z[f"ac_{name}_off"]
    return [z[f"ac_{name}"][off[i]:off[i + 1]] for i in range(off.shape[0] - 1)]


def test_oracle_accumulator_vs_golden(ac):
    acc = O.RelationAccumulator()
    best = [acc.add_row(t, tr, b) for t, tr, b in zip(_rows(ac, "tails"), _rows(ac, "true"), _rows(ac, "base"))]
    np.testing.assert_array_equal(best, ac["ac_best"])
    assert acc.counters() == ac["ac_counters"].tolist()


def _batched(ac, device, split=None):
    from minikg_dev_b200.decode_accum import DecodeAccumulator
    tails, true, base = _rows(ac, "tails"), _rows(ac, "true"), _rows(ac, "base")
    acc = DecodeAccumulator(device)
    best_all = []
    idx = list(range(len(tails)))
    for chunk in ([idx] if split is None else [idx[i:i + split] for i in range(0, len(idx), split)]):
        K = max([1] + [tails[i].size for i in chunk])
        t = np.full((len(chunk), K), -1, np.int64)
        for j, i in enumerate(chunk):
            t[j, :tails[i].size] = tails[i]
        cnt = np.array([tails[i].size for i in chunk], np.int64)
        tp = np.cumsum([0] + [true[i].size for i in chunk]).astype(np.int64)
        bp = np.cumsum([0] + [base[i].size for i in chunk]).astype(np.int64)
        tv = np.concatenate([true[i] for i in chunk]) if chunk else np.zeros(0, np.int64)
        bv = np.concatenate([base[i] for i in chunk]) if chunk else np.zeros(0, np.int64)
        T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(device)  # noqa: E731
        best_all += acc.add_rows(T(t), T(cnt), T(tp), T(tv), T(bp), T(bv)).cpu().tolist()
    return best_all, acc


@pytest.mark.parametrize("split", [None, 7])
def test_batched_accumulator_host_tensors(ac, split):
    best, acc = _batched(ac, "cpu", split)
    np.testing.assert_array_equal(best, ac["ac_best"])
    assert acc.counters == ac["ac_counters"].tolist()
    r = acc.row(3, 100, 40, 60)
    assert r["generated"] == 40 + acc.counters[5] and r["missing"] == 100 - 40 - acc.counters[6]


@pytest.mark.gpu
@pytest.mark.parametrize("split", [None, 7])
def test_batched_accumulator_device(ac, split):
    best, acc = _batched(ac, "cuda", split)
    np.testing.assert_array_equal(best, ac["ac_best"])
    assert acc.counters == ac["ac_counters"].tolist()
