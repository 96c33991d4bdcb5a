"""The C-ABI library builds for sm_100a, loads, exports every declared symbol, and its
ctypes structs match the C layout (no GPU needed: nothing here launches a kernel)."""
from __future__ import annotations

import ctypes
import re
import subprocess
import textwrap
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "minikg_b200.h"


@pytest.fixture(scope="module")
def lib():
    from minikg_dev_b200.build import build
    build()
    from minikg_dev_b200 import _native
    return _native.load()


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mkg_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_bound_set():
    from minikg_dev_b200 import _native
    assert declared_functions() == sorted(_native.SIGNATURES)


def test_every_declared_symbol_is_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(ROOT / "minikg_dev_b200/_lib/libminikg_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(lib, name)
    # nothing else leaks out of the library's namespace
    assert not [s for s in exported if s.startswith("_ZN3mkg")]


def test_library_targets_sm100a():
    out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True).stdout
    assert "12.9" in out
    objs = list((ROOT / "_build").glob("*.o"))
    assert objs, "build() produced no objects"
    from minikg_dev_b200.build import ARCH
    assert "arch=compute_100a,code=sm_100a" in ARCH


STRUCTS = {
    "mkg_csr_dir": ("CsrDir", ["row_ptr", "col_ind", "r_ind", "order", "row_group_ptr", "group_rel",
                               "group_edge_start", "group_edge_count", "num_groups"]),
    "mkg_graph": ("Graph", ["num_entities", "num_relations", "num_facts", "ori", "inv"]),
    "mkg_edge_factor": ("EdgeFactor", ["mask", "mask_kind", "mask_numel", "edge_weight", "edge_weight_numel",
                                       "is_score", "scale"]),
    "mkg_frontier": ("Frontier", ["batch", "level", "entity", "value", "nnz"]),
    "mkg_coo3": ("Coo3", ["indices", "values", "nnz"]),
    "mkg_csr_dir_out": ("CsrDirOut", ["row_ptr", "col_ind", "r_ind", "order", "row_group_ptr", "group_rel",
                                      "group_edge_start", "group_edge_count"]),
    "mkg_adjacency": ("Adjacency", ["pull_ptr", "pull", "push_ptr", "push", "pull_tasks", "num_pull_tasks",
                                    "push_tasks", "num_push_tasks"]),
    "mkg_hop_params": ("HopParams", ["B", "L", "E", "r_size", "n", "wot_i", "agg_mode", "topk_edges", "dst_lo",
                                    "dst_hi", "msg_bound", "accum",
                                    "merge_outputs"]),
    "mkg_proof_params": ("ProofParams", ["B", "L", "E", "R", "hops", "topk_edges", "state_threshold", "reserved",
                                         "fwd_events", "bwd_events", "cap_index"]),
    "mkg_cap_index": ("CapIndex", ["cap", "num_slots", "num_groups", "slot_entity", "slot_dir", "slot_group",
                                   "pull_cap", "push_cap", "capped_degree"]),
    "mkg_rule_params": ("RuleParams", ["n", "H", "L", "K", "U", "B", "tau", "reserved"]),
}


def test_ctypes_layout_matches_c(tmp_path):
    from minikg_dev_b200 import _native
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "minikg_b200.h"', "int main(void) {"]
    for cname, (_, fields) in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f in fields:
            lines.append(f'  printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(ln.rsplit(" ", 1) for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                                                           check=True).stdout.splitlines())
    for cname, (pyname, fields) in STRUCTS.items():
        cls = getattr(_native, pyname)
        assert int(got[f"{cname} size"]) == ctypes.sizeof(cls), cname
        for f in fields:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, f"{cname}.{f}"


def test_product_fails_loudly_without_a_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from minikg_dev_b200.graph import build_csr_structure
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        build_csr_structure(torch.zeros(3, dtype=torch.int32), torch.zeros(3, dtype=torch.int32),
                            torch.zeros(3, dtype=torch.int32), 4)
