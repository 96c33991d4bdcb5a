"""ctypes binding of the C ABI in ``include/minikg_b200.h`` (``_lib/libminikg_b200.so``).

Every wrapper passes raw device pointers of torch tensors plus the current CUDA stream,
raises ``RuntimeError`` with ``mkg_last_error()`` on a non-zero status, and never falls
back to another implementation: without the library (or without a GPU) the call fails.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libminikg_b200.so"

MKG_OK = 0
MASK_NONE, MASK_U8, MASK_F32 = 0, 1, 2
SLAB_SKIP_OUTSIDE = 16  # MKG_SLAB_SKIP_OUTSIDE
SLAB_MAX_TILES = 8  # MKG_SLAB_MAX_TILES
DEV_ERR_NAMES = {1: "frontier entry outside [B, L, E]", 2: "CSR column outside [0, E)",
                 4: "fact id outside [0, T)", 8: "gradient key outside [B, L, E]",
                 16: "relation id outside its range", 32: "a bounded wait inside a kernel gave up",
                 64: "a message hash table ran out of slots (msg_bound too small)",
                 128: "rule producer: relation outside [0, n) or query map outside [0, U)"}

vp = C.c_void_p
i64 = C.c_int64
i32 = C.c_int32


class CsrDir(C.Structure):
    _fields_ = [("row_ptr", vp), ("col_ind", vp), ("r_ind", vp), ("order", vp), ("row_group_ptr", vp),
                ("group_rel", vp), ("group_edge_start", vp), ("group_edge_count", vp), ("num_groups", i64)]


class Graph(C.Structure):
    _fields_ = [("num_entities", i64), ("num_relations", i64), ("num_facts", i64), ("ori", CsrDir),
                ("inv", CsrDir)]


class EdgeFactor(C.Structure):
    _fields_ = [("mask", vp), ("mask_kind", i32), ("mask_numel", i64), ("edge_weight", vp),
                ("edge_weight_numel", i64), ("is_score", i32), ("scale", C.c_float)]


class Frontier(C.Structure):
    _fields_ = [("batch", vp), ("level", vp), ("entity", vp), ("value", vp), ("nnz", i64)]


class Coo3(C.Structure):
    _fields_ = [("indices", vp), ("values", vp), ("nnz", i64)]


class CsrDirOut(C.Structure):
    _fields_ = [("row_ptr", vp), ("col_ind", vp), ("r_ind", vp), ("order", vp), ("row_group_ptr", vp),
                ("group_rel", vp), ("group_edge_start", vp), ("group_edge_count", vp)]


class Adjacency(C.Structure):
    _fields_ = [("pull_ptr", vp), ("pull", vp), ("push_ptr", vp), ("push", vp), ("pull_tasks", vp),
                ("num_pull_tasks", i64), ("push_tasks", vp), ("num_push_tasks", i64)]


class HopParams(C.Structure):
    _fields_ = [("B", i64), ("L", i64), ("E", i64), ("r_size", i64), ("n", i64), ("wot_i", i32),
                ("agg_mode", i32), ("topk_edges", i64), ("dst_lo", i64), ("dst_hi", i64), ("msg_bound", i64),
                ("accum", i64), ("merge_outputs", i64)]


class ProofParams(C.Structure):
    _fields_ = [("B", i64), ("L", i64), ("E", i64), ("R", i64), ("hops", i64), ("topk_edges", i64),
                ("state_threshold", C.c_float), ("reserved", i32), ("fwd_events", vp), ("bwd_events", vp),
                ("cap_index", vp)]


class CapIndex(C.Structure):
    _fields_ = [("cap", i64), ("num_slots", i64), ("num_groups", i64), ("slot_entity", vp), ("slot_dir", vp),
                ("slot_group", vp), ("pull_cap", vp), ("push_cap", vp), ("capped_degree", vp)]


class SlabWindow(C.Structure):
    _fields_ = [("E", i64), ("row0", i64), ("nrows", i64), ("lo", i64), ("extent", i64)]


class RuleParams(C.Structure):
    _fields_ = [("n", i64), ("H", i64), ("L", i64), ("K", i64), ("U", i64), ("B", i64), ("tau", C.c_float),
                ("reserved", i32)]


P = C.POINTER
# name -> (restype, argtypes); every name here must be exported by the library
SIGNATURES = {
    "mkg_last_error": (C.c_char_p, []),
    "mkg_abi_version": (C.c_int, []),
    "mkg_csr_build_workspace_bytes": (C.c_size_t, [i64, i64, i64]),
    "mkg_csr_build": (C.c_int, [vp, vp, vp, i64, i64, i64, CsrDirOut, CsrDirOut, vp, vp, C.c_size_t, vp, vp]),
    "mkg_ind2ptr_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_ind2ptr": (C.c_int, [vp, i64, i64, vp, vp, C.c_size_t, vp, vp]),
    "mkg_ind2ptr_noalloc": (C.c_int, [vp, i64, i64, vp, vp, vp]),
    "mkg_fact_table": (C.c_int, [P(Graph), vp, vp, vp, vp, vp]),
    "mkg_adjacency_max_tasks": (i64, [i64, i64]),
    "mkg_adjacency_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_adjacency_build": (C.c_int, [P(Graph), Adjacency, vp, vp, C.c_size_t, vp, vp]),
    "mkg_adjacency_set_factor": (C.c_int, [P(Graph), Adjacency, P(EdgeFactor), vp]),
    "mkg_records_set_factor": (C.c_int, [vp, i64, i64, P(EdgeFactor), vp]),
    "mkg_hop_forward_workspace_bytes": (C.c_size_t, [P(HopParams), i64]),
    "mkg_hop_forward": (C.c_int, [P(Graph), P(Frontier), vp, P(EdgeFactor), P(HopParams), vp, C.c_size_t, vp,
                                  vp, vp]),
    "mkg_hop_emit": (C.c_int, [P(HopParams), i64, vp, C.c_size_t, C.c_int, i64, vp, vp, vp, vp]),
    "mkg_hop_count_messages": (C.c_int, [P(Graph), P(Frontier), P(HopParams), vp, vp, vp]),
    "mkg_hop_backward_workspace_bytes": (C.c_size_t, [P(HopParams), i64]),
    "mkg_hop_backward": (C.c_int, [P(Graph), P(Frontier), vp, P(EdgeFactor), P(HopParams), P(Coo3), P(Coo3),
                                   P(Coo3), P(Coo3), vp, P(Coo3), vp, vp, vp, vp, vp, vp, vp, vp, C.c_size_t,
                                   vp, vp]),
    "mkg_proof_workspace_bytes": (C.c_size_t, [P(ProofParams)]),
    "mkg_proof_forward": (C.c_int, [P(Graph), P(Adjacency), vp, vp, P(ProofParams), vp, C.c_size_t, vp, vp, vp,
                                    vp]),
    "mkg_proof_backward": (C.c_int, [P(Graph), P(Adjacency), vp, P(ProofParams), P(EdgeFactor), vp, vp, vp, vp,
                                     C.c_size_t, vp, vp]),
    "mkg_proof_row_activity": (C.c_int, [P(ProofParams), vp, C.c_size_t, i64, vp, vp]),
    "mkg_decode_workspace_bytes": (C.c_size_t, [P(ProofParams), i64]),
    "mkg_proof_decode_max": (C.c_int, [P(Graph), P(Adjacency), vp, vp, P(ProofParams), i64, vp, vp, vp, vp, vp,
                                       C.c_size_t, vp, vp]),
    "mkg_decode_topk": (C.c_int, [vp, i64, i64, i64, vp, vp, vp, vp]),
    "mkg_sparse_topk_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_sparse_topk": (C.c_int, [vp, vp, i64, i64, i64, i64, vp, vp, vp, vp, C.c_size_t, vp]),
    "mkg_segment_sum_ordered": (C.c_int, [vp, i64, vp, vp, vp]),
    "mkg_segment_sum": (C.c_int, [vp, i64, vp, vp, vp]),
    "mkg_cap_index_workspace_bytes": (C.c_size_t, [P(Graph)]),
    "mkg_cap_index_sizes": (C.c_int, [P(Graph), i64, vp, vp, C.c_size_t, vp]),
    "mkg_cap_index_build": (C.c_int, [P(Graph), P(Adjacency), P(CapIndex), vp, C.c_size_t, vp, vp]),
    "mkg_slab_store_bytes": (C.c_size_t, [i64]),
    "mkg_slab_expand_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_slab_expand": (C.c_int, [vp, vp, vp, vp, i64, vp, i64, i32, i32, P(SlabWindow), vp, vp, vp, C.c_size_t,
                                  vp, vp]),
    "mkg_slab_expand_tiles": (C.c_int, [i32, vp, vp, vp, vp, i64, vp, i64, i32, i32, P(SlabWindow), vp, vp, vp,
                                        C.c_size_t, vp, vp]),
    "mkg_slab_collect_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_slab_count": (C.c_int, [P(SlabWindow), vp, vp, C.c_size_t, vp, vp]),
    "mkg_slab_emit": (C.c_int, [P(SlabWindow), vp, vp, C.c_size_t, i64, vp, vp, vp]),
    "mkg_slab_emit_normalized": (C.c_int, [P(SlabWindow), vp, vp, C.c_size_t, i64, vp, C.c_float, vp, vp, vp, vp,
                                           vp]),
    "mkg_slab_put": (C.c_int, [P(SlabWindow), vp, vp, vp, i64, i64, i32, vp, vp]),
    "mkg_slab_take": (C.c_int, [P(SlabWindow), vp, vp, i64, i64, vp, i32, vp, vp]),
    "mkg_slab_expand_backward": (C.c_int, [vp, vp, vp, vp, i64, vp, i64, i32, P(SlabWindow), vp, P(EdgeFactor),
                                           i64, vp, vp, vp, vp, C.c_size_t, vp, vp]),
    "mkg_slab_expand_backward_tiles": (C.c_int, [i32, vp, vp, vp, vp, i64, vp, i64, i32, P(SlabWindow), vp,
                                                 P(EdgeFactor), i64, vp, vp, vp, vp, C.c_size_t, vp, vp]),
    "mkg_row_sums": (C.c_int, [vp, i64, i64, i64, i64, vp, vp, vp, vp]),
    "mkg_f64_to_f32": (C.c_int, [vp, i64, vp, vp]),
    "mkg_mass_normalize": (C.c_int, [vp, vp, i64, i64, i64, i64, vp, C.c_float, vp, vp, vp, vp]),
    "mkg_mass_normalize_grad_sums": (C.c_int, [vp, vp, vp, i64, i64, i64, i64, vp, vp, vp, vp]),
    "mkg_mass_normalize_grad": (C.c_int, [vp, vp, vp, i64, i64, i64, i64, vp, vp, vp, vp]),
    "mkg_mass_normalize_grad_put": (C.c_int, [vp, vp, vp, i64, i64, i64, i64, vp, vp, P(SlabWindow), vp, vp, vp]),
    "mkg_rule_sum_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_rule_sum": (C.c_int, [vp, vp, i64, i64, i64, i64, i32, vp, vp, vp, vp, vp, C.c_size_t, vp, vp]),
    "mkg_reduce_by_key_workspace_bytes": (C.c_size_t, [i64]),
    "mkg_reduce_by_key": (C.c_int, [vp, vp, i64, i32, i32, vp, vp, vp, vp, vp, vp, C.c_size_t, vp, vp]),
    "mkg_rule_saved_bytes": (C.c_size_t, [P(RuleParams)]),
    "mkg_rule_backward_workspace_bytes": (C.c_size_t, [P(RuleParams)]),
    "mkg_rule_softmax_workspace_bytes": (C.c_size_t, [P(RuleParams)]),
    "mkg_rule_logits_forward": (C.c_int, [P(RuleParams), vp, vp, vp, vp, vp, vp, vp, vp, vp, C.c_size_t, vp,
                                          vp]),
    "mkg_rule_logits_backward": (C.c_int, [P(RuleParams), vp, vp, vp, vp, vp, vp, C.c_size_t, vp, vp, vp, vp, vp,
                                           vp, vp, vp, C.c_size_t, vp, vp]),
    "mkg_rule_softmax_forward": (C.c_int, [P(RuleParams), vp, vp, vp, vp, vp]),
    "mkg_rule_softmax_backward": (C.c_int, [P(RuleParams), vp, vp, vp, vp, vp, vp, C.c_size_t, vp, vp]),
}

_lib = None
_lock = threading.Lock()


def load(path: Path | str | None = None):
    """Loads (once) and returns the library; raises if it was not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(f"minikg_b200 native library missing at {p}; run "
                               "`python -m minikg_dev_b200.build` (nvcc, sm_100a)")
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def last_error() -> str:
    msg = load().mkg_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status != MKG_OK:
        raise RuntimeError(f"minikg_b200 {what} failed (status {status}): {last_error()}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"minikg_b200: {what} must be a CUDA tensor (the library has no CPU path)")


_err_words: dict[int, torch.Tensor] = {}


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 error word the kernels OR their MKG_DEV_* bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _err_words.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_words[idx] = w
    return w


def raise_device_errors(device: torch.device) -> None:
    """Synchronises with the error word; raises (and clears it) if a kernel flagged a bad index."""
    w = error_word(device)
    bits = int(w.item())
    if bits:
        w.zero_()
        names = [v for k, v in DEV_ERR_NAMES.items() if bits & k]
        raise RuntimeError("minikg_b200 kernel rejected its input: " + "; ".join(names))


def segment_sum(seg_ptr: torch.Tensor, values: torch.Tensor, ordered: bool = False) -> torch.Tensor:
    """Per-segment sums of ``values`` (``seg_ptr`` int64 [nseg + 1], device tensors);
    ``ordered``: each segment added one by one in index order (bit-reproducible)."""
    v = values.detach().to(torch.float32).contiguous()
    sp = seg_ptr.to(torch.int64).contiguous()
    nseg = int(sp.numel()) - 1
    out = torch.empty(max(nseg, 0), dtype=torch.float32, device=v.device)
    fn = load().mkg_segment_sum_ordered if ordered else load().mkg_segment_sum
    check(fn(sp.data_ptr(), nseg, v.data_ptr(), out.data_ptr(), stream_handle(v.device)), "segment_sum")
    return out


def row_sums(keys: torch.Tensor, values: torch.Tensor, E: int, nrows: int, row0: int = 0) -> torch.Tensor:
    """fp64 [nrows]: the sum of ``values`` over each row ``key // E - row0`` of the ascending
    ``keys`` (int64 device tensors), accumulated in fp64."""
    k = keys.to(torch.int64).contiguous()
    v = values.detach().to(torch.float32).contiguous()
    out = torch.zeros(max(int(nrows), 1), dtype=torch.float64, device=v.device)
    check(load().mkg_row_sums(k.data_ptr(), int(k.numel()), int(E), int(row0), int(nrows), v.data_ptr(),
                              out.data_ptr(), error_word(v.device).data_ptr(), stream_handle(v.device)), "row_sums")
    return out[: int(nrows)]


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def edge_factor(mask: torch.Tensor | None, weight: torch.Tensor | None, is_score: bool, scale: float,
                keep: list) -> EdgeFactor:
    """Builds the factor struct; tensors it points to are appended to ``keep``."""
    f = EdgeFactor()
    if mask is None:
        f.mask, f.mask_kind, f.mask_numel = None, MASK_NONE, 0
    else:
        m = mask.reshape(-1)
        if m.dtype == torch.bool or m.dtype == torch.uint8:
            m = m.contiguous().view(torch.uint8) if m.dtype == torch.bool else m.contiguous()
            kind = MASK_U8
        else:
            m = m.to(torch.float32).contiguous()
            kind = MASK_F32
        keep.append(m)
        f.mask, f.mask_kind, f.mask_numel = m.data_ptr(), kind, m.numel()
    if weight is None or weight.numel() == 0:
        f.edge_weight, f.edge_weight_numel = None, 0
    else:
        wt = weight.detach().reshape(-1).to(torch.float32).contiguous()
        keep.append(wt)
        f.edge_weight, f.edge_weight_numel = wt.data_ptr(), wt.numel()
    f.is_score = 1 if is_score else 0
    f.scale = float(scale)
    return f
