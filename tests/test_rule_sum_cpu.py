"""The written-out fold that ``test_slab_gpu.test_rule_sum_entity_major`` holds ``mkg_rule_sum``
to, pinned on the CPU to the oracle's ``sum_sp_3d`` / ``max_sp_3d`` (fastlog_bridge.py:17-23,
model_mmDRUM_kernel_sp.py:184-211): the same keys, bit-identical values (fp32 sums in rule order;
maxima), and each entry's reported result index pointing at its own (b, e) key."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import fastlog_oracle as O
from tests.test_slab_gpu import _rule_sum_reference


def _entity_major_state(E, B, L, n, seed):
    """About n entries: (e, b) pairs, each with a random non-empty subset of its L rules, in
    entity-major order (ascending entity, then row b * L + l), the slab emit's order."""
    rng = np.random.default_rng(seed)
    m = min(E * B, max(1, int(n / (0.7 * L + 0.3))))
    pairs = rng.choice(E * B, size=m, replace=False).astype(np.int64)
    take = rng.random((m, L)) < 0.7
    take[np.arange(m), rng.integers(0, L, m)] = True
    ii, ll = np.nonzero(take)
    keys = (pairs[ii] % B * L + ll) * E + pairs[ii] // B
    keys = keys[np.lexsort((keys // E, keys % E))].astype(np.int64)
    return keys, rng.uniform(0.01, 1.0, keys.size).astype(np.float32)


@pytest.mark.parametrize("E,B,L,n", [(500, 30, 4, 3000), (90, 3, 2, 500), (400, 1, 1, 300), (200, 1500, 3, 2000)])
def test_rule_sum_fold_matches_oracle(E, B, L, n):
    keys, vals = _entity_major_state(E, B, L, n, seed=E + B)
    rk, rv, rpos = _rule_sum_reference(keys, vals, E, L, take_max=False)
    ok, ov = O.sum_sp_3d((keys, vals), L, E)
    np.testing.assert_array_equal(rk, ok)
    np.testing.assert_array_equal(rv.view(np.uint32), ov.astype(np.float32).view(np.uint32))
    mk, mv, mpos = _rule_sum_reference(keys, vals, E, L, take_max=True)
    ok2, ov2 = O.max_sp_3d((keys, vals), L, E)  # (positive values: no zero is dropped)
    np.testing.assert_array_equal(mk, ok2)
    np.testing.assert_array_equal(mv.view(np.uint32), ov2.astype(np.float32).view(np.uint32))
    own = ((keys // E) // L) * E + keys % E
    np.testing.assert_array_equal(rk[rpos], own)
    np.testing.assert_array_equal(mk[mpos], own)
