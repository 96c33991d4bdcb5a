"""mkg_ind2ptr_noalloc: ind2ptr without any device allocation, for callers that cannot
allocate (a C / FFI host that only holds the device pointers it was given).

It is called through the C ABI exactly as such a caller would, and its output is checked
against the workspace-based mkg_ind2ptr on the same inputs, on two calls in a row (the
second smaller than the first, so counts left in the shared static scratch by the first
call would show up if they were not cleared).  The file sorts last so that a failure here
comes after every other test has run.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _with_workspace(lib, N, idx, size, dev):
    out = torch.empty(size + 1, dtype=torch.int64, device=dev)
    ws = N.workspace(lib.mkg_ind2ptr_workspace_bytes(size), dev)
    N.check(lib.mkg_ind2ptr(idx.data_ptr(), idx.numel(), size, out.data_ptr(), ws.data_ptr(), ws.numel(),
                            N.error_word(dev).data_ptr(), N.stream_handle(dev)), "ind2ptr")
    return out


def _no_alloc(lib, N, idx, size, dev):
    out = torch.empty(size + 1, dtype=torch.int64, device=dev)
    N.check(lib.mkg_ind2ptr_noalloc(idx.data_ptr(), idx.numel(), size, out.data_ptr(),
                                    N.error_word(dev).data_ptr(), N.stream_handle(dev)), "ind2ptr_noalloc")
    return out


def test_ind2ptr_noalloc_matches_workspace_version():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from minikg_dev_b200 import _native as N
    lib = N.load()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(2024)
    cases = [(900_000, 250_000), (5_000, 3_000)]  # second call smaller than the first
    for size, n in cases:
        idx = torch.from_numpy(np.sort(rng.integers(0, size, n))).to(dev)
        got = _no_alloc(lib, N, idx, size, dev)
        want = _with_workspace(lib, N, idx, size, dev)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert int(got[-1].item()) == n
    N.raise_device_errors(dev)


def test_ind2ptr_noalloc_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from minikg_dev_b200 import _native as N
    lib = N.load()
    dev = torch.device("cuda", 0)
    size = (1 << 20) + 1
    idx = torch.zeros(4, dtype=torch.int64, device=dev)
    out = torch.empty(size + 1, dtype=torch.int64, device=dev)
    rc = lib.mkg_ind2ptr_noalloc(idx.data_ptr(), idx.numel(), size, out.data_ptr(), None, N.stream_handle(dev))
    assert rc == 3  # MKG_ERR_CAPACITY, reported on the host before any launch
    assert "static scratch limit" in N.last_error()
    assert ctypes.c_int(rc).value != 0
