"""The per-hop operator behind the reference's ``fastlog_bridge`` API, on the B200 library.

``FastLogFunctionSparse3DTopK`` keeps the reference signature, argument meaning, tuple
order and return values (src/fastlog_kernel/fastlog_kernel.py:900-1107): three coalesced
sparse COO ``[B, L, E]`` tensors (ori, inv, ind), and gradients for ``sp_value``, ``w`` and
the edge weights.  Forward and backward each run in the C library (``mkg_hop_forward`` /
``mkg_hop_emit`` / ``mkg_hop_backward``); raw messages are never materialised and no torch
sort-coalesce runs.

Semantics kept from the reference's CUDA path:
* edge factor ``bool(mask[f]) * score(f)``; messages with a zero factor still create their
  output key (explicit zeros), as the fill kernel does (fastlog.cu:2300-2318);
* the 256-bucket per-entry edge cap with in-order threshold groups;
* ``agg_mode == 1``: max per key, argmax = smallest original fact id among equal maxima
  (``tie_break=meta_edge``, fastlog_kernel.py:954-959); the backward sends each key's
  gradient to that message only.
Reference environment flags kept: ``FASTLOG_STAGE_TIMING=1`` prints ``StageTiming`` lines per
stage (prepare_inputs, cuda_forward — which here includes the coalescing —, save_ctx);
``FASTLOG_SPARSE_DEBUG_COUNTS=1`` prints the raw message counts (``Sparse3DTopKCounts``);
``FASTLOG_SPARSE_EDGE_GRAD=1`` returns the edge-score gradient as sparse COO.
Differences: a ``mask_values`` of one element (the reference's 0-d ones tensor for huge
graphs) is broadcast to every fact; the max path compares values through an
order-preserving integer key, so ``-0.0`` ranks below ``+0.0``.
"""
from __future__ import annotations

import ctypes
import os
import time

import torch
from torch import autograd

from . import _native as N
from .graph import build_csr_structure, graph_from_csr  # noqa: F401  (re-exported)


def _stage_timing() -> bool:
    return os.environ.get("FASTLOG_STAGE_TIMING", "") == "1"


def _stage_log(stage: str, t0: float) -> None:
    """``FASTLOG_STAGE_TIMING=1``: one line per op stage after a device sync, in the reference's
    format (fastlog_kernel.py:50-66)."""
    if not _stage_timing():
        return
    if torch.cuda.is_available():
        torch.cuda.synchronize()
    print("StageTiming fastlog_kernel stage:{} seconds:{:.4f}".format(stage, time.perf_counter() - float(t0)))


# Message store of the op: "auto" (key spaces above _HASH_MIN_KEYS count their messages -- one
# extra host sync per hop -- and take hash tables when the count is far below the key space),
# "dense" (always the key slab) or "hash" (always hash tables).
ACCUM = "auto"
ACCUM_MODES = {"auto": 0, "dense": 1, "hash": 2}
_HASH_MIN_KEYS = 1 << 24


def _frontier(sp_batch, sp_level, sp_entity, sp_value, keep):
    b = sp_batch.to(torch.int64).contiguous()
    l = sp_level.to(torch.int64).contiguous()
    e = sp_entity.to(torch.int64).contiguous()
    v = sp_value.detach().to(torch.float32).contiguous()
    keep += [b, l, e, v]
    return N.Frontier(b.data_ptr(), l.data_ptr(), e.data_ptr(), v.data_ptr(), b.numel()), (b, l, e, v)


def _coo(t: torch.Tensor | None, B, L, E, like_indices: torch.Tensor | None, keep):
    """(indices [3, nnz] int64, values fp32) of a gradient; dense gradients are read at the
    forward output's keys (the only keys any message reached)."""
    if t is None:
        z = torch.empty((3, 0), dtype=torch.int64, device=like_indices.device if like_indices is not None else "cuda")
        v = torch.empty(0, dtype=torch.float32, device=z.device)
    elif t.is_sparse:
        t = t.coalesce()
        z = t.indices().to(torch.int64).contiguous()
        v = t.values().to(torch.float32).contiguous()
    else:
        z = like_indices.contiguous()
        v = t[z[0], z[1], z[2]].to(torch.float32).contiguous()
    keep += [z, v]
    return N.Coo3(z.data_ptr(), v.data_ptr(), int(v.numel()))


def _hop_forward(ctx, g, sp_batch, sp_level, sp_entity, sp_value, w, mask_values, weight, B, L, r_size, wot_i,
                 topk_edges, agg_mode, edge_weight_is_score, edge_weight_scale, dst_lo=0, dst_hi=0):
    """Forward of one hop on a ``DeviceGraph``; outputs hold the keys with e in [dst_lo, dst_hi)
    (the whole [0, E) when dst_hi <= dst_lo)."""
    t_stage = time.perf_counter()
    lib = N.load()
    N.require_cuda(sp_value, "sp_value")
    dev = sp_value.device
    B, L, E, r_size = int(B), int(L), int(g.num_entities), int(r_size)
    keep = []
    fr, (b, l, e, v) = _frontier(sp_batch, sp_level, sp_entity, sp_value, keep)
    wf = w.detach().to(torch.float32).contiguous()
    if wf.dim() != 3 or wf.shape[0] != B or wf.shape[1] != L:
        raise ValueError(f"w must be [B, L, n], got {tuple(wf.shape)}")
    n = int(wf.shape[2])
    edge_weight = weight if (weight is not None and weight.numel() > 0) else None
    f = N.edge_factor(mask_values, edge_weight, bool(edge_weight_is_score), float(edge_weight_scale), keep)
    params = [B, L, E, r_size, n, 1 if wot_i else 0, int(agg_mode), int(topk_edges), int(dst_lo), int(dst_hi), 0,
              ACCUM_MODES[ACCUM], 0]
    p = N.HopParams(*params)
    nnz = int(b.numel())
    extent = (int(dst_hi) - int(dst_lo)) if int(dst_hi) > int(dst_lo) else E
    _stage_log("sparse3d_topk.prepare_inputs", t_stage)
    t_stage = time.perf_counter()
    debug_counts = os.environ.get("FASTLOG_SPARSE_DEBUG_COUNTS", "") == "1"
    if debug_counts:
        # the reference's raw message counts (fastlog_kernel.py:940-949): ori / inv messages
        # before coalescing, one identity message per entry
        mcd = torch.empty(2, dtype=torch.int64, device=dev)
        N.check(lib.mkg_hop_count_messages(ctypes.byref(g.struct), ctypes.byref(fr), ctypes.byref(p), mcd.data_ptr(),
                                           N.error_word(dev).data_ptr(), N.stream_handle(dev)), "hop_count_messages")
        m_ori, m_inv = (int(x) for x in mcd.tolist())
        print("Sparse3DTopKCounts nnz={} ori_total={} inv_total={} ind_total={}".format(nnz, m_ori, m_inv, nnz),
              flush=True)
    if ACCUM == "hash" or (ACCUM == "auto" and B * L * extent > _HASH_MIN_KEYS):
        # exact message counts decide between the dense key slab and hash tables
        mc = torch.empty(2, dtype=torch.int64, device=dev)
        N.check(lib.mkg_hop_count_messages(ctypes.byref(g.struct), ctypes.byref(fr), ctypes.byref(p), mc.data_ptr(),
                                           N.error_word(dev).data_ptr(), N.stream_handle(dev)), "hop_count_messages")
        params[10] = max(1, int(mc.max().item()))
        p = N.HopParams(*params)
    params = tuple(params)
    ws = N.workspace(lib.mkg_hop_forward_workspace_bytes(ctypes.byref(p), nnz), dev)
    counts = torch.zeros(3, dtype=torch.int64, device=dev)
    err = N.error_word(dev)
    st = N.stream_handle(dev)
    N.check(lib.mkg_hop_forward(ctypes.byref(g.struct), ctypes.byref(fr), wf.data_ptr(), ctypes.byref(f),
                                ctypes.byref(p), ws.data_ptr(), ws.numel(), counts.data_ptr(), err.data_ptr(), st),
            "hop_forward")
    sizes = counts.tolist()  # the one host sync of the hop (the reference has one too)
    N.raise_device_errors(dev)
    outs, args = [], []
    for which, U in enumerate(sizes):
        idx = torch.empty((3, U), dtype=torch.int64, device=dev)
        val = torch.empty(U, dtype=torch.float32, device=dev)
        arg = torch.empty(U, dtype=torch.int64, device=dev) if (agg_mode == 1 and which < 2) else None
        N.check(lib.mkg_hop_emit(ctypes.byref(p), nnz, ws.data_ptr(), ws.numel(), which, U, idx.data_ptr(),
                                 val.data_ptr(), arg.data_ptr() if arg is not None else None, st), "hop_emit")
        outs.append(torch.sparse_coo_tensor(idx, val, (B, L, E), is_coalesced=True))
        args.append(arg)
    del ws
    _stage_log("sparse3d_topk.cuda_forward", t_stage)
    t_stage = time.perf_counter()
    has_edge_weight = weight is not None and bool(getattr(weight, "requires_grad", False))
    if any(ctx.needs_input_grad):
        empty_i = torch.empty(0, dtype=torch.int64, device=dev)
        saved = [b, l, e, v, wf, outs[0]._indices(), outs[1]._indices(), outs[2]._indices()]
        saved += [args[0] if args[0] is not None else empty_i, args[1] if args[1] is not None else empty_i]
        saved += [mask_values if mask_values is not None else torch.empty(0, device=dev)]
        saved += [weight.detach() if edge_weight is not None else torch.empty(0, device=dev)]
        ctx.save_for_backward(*saved)
        ctx.g = g
        ctx.params = params
        ctx.has_mask = mask_values is not None
        ctx.has_edge_weight = has_edge_weight
        ctx.edge_weight_present = edge_weight is not None
        ctx.edge_weight_is_score = bool(edge_weight_is_score)
        ctx.edge_weight_scale = float(edge_weight_scale)
        ctx.weight_shape = tuple(weight.shape) if weight is not None else None
        ctx.weight_dtype = weight.dtype if weight is not None else None
    _stage_log("sparse3d_topk.save_ctx", t_stage)
    return outs[0], outs[1], outs[2]


def _hop_backward(ctx, grad_ori, grad_inv, grad_ind):
    """(grad_sp, grad_w, grad_edge_weight) of ``_hop_forward``."""
    lib = N.load()
    b, l, e, v, wf, oi_ori, oi_inv, oi_ind, arg_ori, arg_inv, mask_values, weight = ctx.saved_tensors
    B, L, E, r_size, n, wot_i, agg_mode, topk, dst_lo, dst_hi, msg_bound, accum, merge = ctx.params
    g = ctx.g
    dev = v.device
    keep = []
    fr = N.Frontier(b.data_ptr(), l.data_ptr(), e.data_ptr(), v.data_ptr(), b.numel())
    f = N.edge_factor(mask_values if ctx.has_mask else None, weight if ctx.edge_weight_present else None,
                      ctx.edge_weight_is_score, ctx.edge_weight_scale, keep)
    p = N.HopParams(*ctx.params)
    go = _coo(grad_ori, B, L, E, oi_ori, keep)
    gi = _coo(grad_inv, B, L, E, oi_inv, keep)
    gd = _coo(grad_ind, B, L, E, oi_ind, keep)
    grad_sp = torch.empty(b.numel(), dtype=torch.float32, device=dev)
    grad_w = torch.empty((B, L, n), dtype=torch.float32, device=dev)
    grad_edge = torch.empty(g.num_facts, dtype=torch.float32, device=dev) if ctx.has_edge_weight else None
    out_o = N.Coo3(oi_ori.data_ptr(), None, int(oi_ori.shape[1]))
    out_i = N.Coo3(oi_inv.data_ptr(), None, int(oi_inv.shape[1]))
    fh = ft = frl = None
    if agg_mode == 1:
        fh, ft, frl = g.fact_table()
    ws = N.workspace(lib.mkg_hop_backward_workspace_bytes(ctypes.byref(p), b.numel()), dev)
    N.check(lib.mkg_hop_backward(ctypes.byref(g.struct), ctypes.byref(fr), wf.data_ptr(), ctypes.byref(f),
                                 ctypes.byref(p), ctypes.byref(go), ctypes.byref(gi), ctypes.byref(gd),
                                 ctypes.byref(out_o), N.ptr(arg_ori) if arg_ori.numel() else None,
                                 ctypes.byref(out_i), N.ptr(arg_inv) if arg_inv.numel() else None,
                                 N.ptr(fh), N.ptr(ft), N.ptr(frl), grad_sp.data_ptr(), grad_w.data_ptr(),
                                 N.ptr(grad_edge), ws.data_ptr(), ws.numel(), N.error_word(dev).data_ptr(),
                                 N.stream_handle(dev)), "hop_backward")
    grad_edge_weight = None
    if ctx.has_edge_weight:
        if os.environ.get("FASTLOG_SPARSE_EDGE_GRAD", "0") == "1":
            nz = torch.nonzero(grad_edge, as_tuple=True)[0]
            if len(ctx.weight_shape) == 2 and ctx.weight_shape[1] == 1:
                idx = torch.stack([nz, torch.zeros_like(nz)])
            else:
                idx = nz.view(1, -1)
            grad_edge_weight = torch.sparse_coo_tensor(idx, grad_edge[nz].to(ctx.weight_dtype),
                                                       ctx.weight_shape, device=dev).coalesce()
        else:
            grad_edge_weight = grad_edge.view(ctx.weight_shape).to(ctx.weight_dtype)
    return grad_sp.to(v.dtype), grad_w, grad_edge_weight


class FastLogFunctionSparse3DTopK(autograd.Function):
    """One relation-typed hop (reference: fastlog_kernel.py:900-1107)."""

    @staticmethod
    def forward(ctx, sp_batch, sp_level, sp_entity, sp_value, w,
                ori_row_ptr, ori_col_ind, ori_r_ind, ori_order,
                inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
                ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
                inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count,
                mask_values, weight, B, L, E, r_size, wot_i, topk_edges, agg_mode=0,
                edge_weight_is_score=False, edge_weight_scale=1.0):
        csr = (ori_row_ptr, ori_col_ind, ori_r_ind, ori_order, inv_row_ptr, inv_col_ind, inv_r_ind, inv_order,
               ori_row_group_ptr, ori_group_rel, ori_group_edge_start, ori_group_edge_count,
               inv_row_group_ptr, inv_group_rel, inv_group_edge_start, inv_group_edge_count)
        g = graph_from_csr(csr, int(E), int(r_size))
        return _hop_forward(ctx, g, sp_batch, sp_level, sp_entity, sp_value, w, mask_values, weight, B, L, r_size,
                            wot_i, topk_edges, agg_mode, edge_weight_is_score, edge_weight_scale)

    @staticmethod
    def backward(ctx, grad_ori, grad_inv, grad_ind):
        grad_sp, grad_w, grad_edge_weight = _hop_backward(ctx, grad_ori, grad_inv, grad_ind)
        return (None, None, None, grad_sp, grad_w,
                None, None, None, None,
                None, None, None, None,
                None, None, None, None,
                None, None, None, None,
                None, grad_edge_weight,
                None, None, None, None, None, None, None, None, None)


class HopRange(autograd.Function):
    """One hop on a resident ``DeviceGraph`` restricted to destinations in [dst_lo, dst_hi):
    ``(ori, inv, ind)`` hold only those keys (shape [B, L, E]); caps are decided on whole
    CSR rows, so the outputs over a partition of [0, E) add up to the full-range op.
    Gradients flow to ``sp_value``, ``w`` and ``weight``."""

    @staticmethod
    def forward(ctx, sp_batch, sp_level, sp_entity, sp_value, w, graph, mask_values, weight, B, L, wot_i,
                topk_edges, agg_mode, edge_weight_is_score, edge_weight_scale, dst_lo, dst_hi):
        return _hop_forward(ctx, graph, sp_batch, sp_level, sp_entity, sp_value, w, mask_values, weight, B, L,
                            graph.num_relations, wot_i, topk_edges, agg_mode, edge_weight_is_score,
                            edge_weight_scale, dst_lo, dst_hi)

    @staticmethod
    def backward(ctx, grad_ori, grad_inv, grad_ind):
        grad_sp, grad_w, grad_edge_weight = _hop_backward(ctx, grad_ori, grad_inv, grad_ind)
        return (None, None, None, grad_sp, grad_w, None, None, grad_edge_weight,
                None, None, None, None, None, None, None, None, None)
