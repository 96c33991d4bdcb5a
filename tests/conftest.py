"""Shared pytest setup: the ``gpu`` marker and helpers to load the golden fixtures."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C-ABI")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"golden_{name}.npz") as z:
        return {k: z[k] for k in z.files}


GRAD_RTOL, GRAD_ATOL = 1e-5, 1e-6  # the sum path's bar, for the hop-loop gradients too


def exact_loop_grads(heads, w_hops, csr, mask, scores, B, L, E, R, final_keys, seed, **kw):
    """Rule-weight and edge-score gradients of the oracle's sum hop loop run in float64
    arithmetic (``float64_arithmetic``), for ``seed`` on the fp32 run's final keys.  The CUDA
    loops are held to the fp32 bar against these: over several hops the reference's own fp32
    rounding moves its gradients further than that bar from this value (measured in
    test_oracle_golden.py), so an fp32 oracle run cannot serve as the yardstick at this bar."""
    from oracle import fastlog_oracle as O
    num_facts = kw.pop("num_facts")
    bwd_kw = {k: kw[k] for k in ("is_score", "scale") if k in kw}
    with O.float64_arithmetic():
        final, trace = O.proof_sum_forward(heads, w_hops, csr, mask, scores, B, L, E, R, **kw)
        gw, ge = O.proof_sum_backward(trace, (np.asarray(final_keys, np.int64), np.asarray(seed, np.float64)),
                                      w_hops, csr, mask, scores, B, L, E, R, num_facts=num_facts, **bwd_kw)
    if float(kw.get("threshold", 0.0)) <= 0:  # a state threshold may keep another set near its edge
        np.testing.assert_array_equal(final[0], final_keys)  # same result keys as the fp32 run
    return gw, ge


def softmax_backward(w, g):
    """d loss / d logits of ``w = softmax(logits)`` over the last axis (float64)."""
    w = np.asarray(w, np.float64)
    g = np.asarray(g, np.float64)
    return w * (g - (w * g).sum(axis=-1, keepdims=True))


@pytest.fixture(scope="session", params=["g1", "g2"])
def golden_graph(request):
    return request.param, load_golden(request.param)


@pytest.fixture(scope="session")
def golden_reducers():
    return load_golden("reducers")
