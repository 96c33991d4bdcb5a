"""Drop-in for the reference operator API ``src/fastlog_bridge.py`` (names of ``__all__``,
src/fastlog_bridge.py:45-50), plus the two reducers ``proof.kernel_ops()`` imports from
src/model_mmDRUM_kernel_sp.py (proof.py:42-58)."""
from __future__ import annotations

from .fastlog_kernel import FastLogFunctionSparse3DTopK
from .graph import build_csr_structure
from .sparse_reducers import max_sp_3d, sparse3d_max, sum_sp_3d, sum_sparse3d_concat

__all__ = [
    "FastLogFunctionSparse3DTopK",
    "build_csr_structure",
    "sum_sp_3d",
    "sum_sparse3d_concat",
]


def kernel_ops():
    """The 6-tuple ``proof.kernel_ops()`` returns (proof.py:39-59)."""
    return (FastLogFunctionSparse3DTopK, build_csr_structure, max_sp_3d, sparse3d_max, sum_sp_3d,
            sum_sparse3d_concat)
