"""Device-resident knowledge-graph structures.

``build_csr_structure`` is the drop-in for the reference's
``src/fastlog_kernel/fastlog_kernel.py:371-411``: it returns the same 16-tuple (dtypes
and tuple order of ``:403-410``) but sorts on the GPU (stable radix sort by (row, rel,
fact id)) instead of a host ``argsort``.  ``DeviceGraph`` wraps such a tuple together with
the structures the fused hop loop needs (merged pull / push neighbour lists cut into
tasks, and the per-fact endpoint table of the argmax backward), built once per graph.
"""
from __future__ import annotations

from collections import OrderedDict

import torch

from . import _native as N

CSR_DTYPES = (torch.int32, torch.int32, torch.int16, torch.int32,
              torch.int32, torch.int32, torch.int16, torch.int32,
              torch.int32, torch.int16, torch.int32, torch.int32,
              torch.int32, torch.int16, torch.int32, torch.int32)


def build_csr_structure(row_indices: torch.Tensor, col_indices: torch.Tensor, r_indices: torch.Tensor,
                        num_nodes: int, num_relations: int | None = None):
    """Both CSR directions of the graph (rows = head for ori, tail for inv).

    Same arguments and 16-tuple as the reference (fastlog_kernel.py:371-411); inputs must
    be CUDA tensors.  Within one (row, relation) group facts keep ascending fact-id order
    (the reference's ``torch.argsort`` leaves that order unspecified).
    """
    lib = N.load()
    N.require_cuda(row_indices, "row_indices")
    dev = row_indices.device
    head = row_indices.to(torch.int32).contiguous()
    tail = col_indices.to(device=dev, dtype=torch.int32).contiguous()
    rel = r_indices.to(device=dev, dtype=torch.int32).contiguous()
    T = int(head.numel())
    E = int(num_nodes)
    if T == 0:
        z = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        e32 = torch.empty(0, dtype=torch.int32, device=dev)
        e16 = torch.empty(0, dtype=torch.int16, device=dev)
        return (z, e32, e16, e32, z.clone(), e32, e16, e32, z.clone(), e16, e32, e32, z.clone(), e16, e32, e32)
    R = int(num_relations) if num_relations is not None else int(rel.max().item()) + 1
    outs = []
    structs = []
    for _ in range(2):
        o = dict(row_ptr=torch.empty(E + 1, dtype=torch.int32, device=dev),
                 col_ind=torch.empty(T, dtype=torch.int32, device=dev),
                 r_ind=torch.empty(T, dtype=torch.int16, device=dev),
                 order=torch.empty(T, dtype=torch.int32, device=dev),
                 row_group_ptr=torch.empty(E + 1, dtype=torch.int32, device=dev),
                 group_rel=torch.empty(T, dtype=torch.int16, device=dev),
                 group_edge_start=torch.empty(T, dtype=torch.int32, device=dev),
                 group_edge_count=torch.empty(T, dtype=torch.int32, device=dev))
        outs.append(o)
        structs.append(N.CsrDirOut(*[o[k].data_ptr() for k in ("row_ptr", "col_ind", "r_ind", "order",
                                                              "row_group_ptr", "group_rel", "group_edge_start",
                                                              "group_edge_count")]))
    ngroups = torch.zeros(2, dtype=torch.int64, device=dev)
    ws = N.workspace(lib.mkg_csr_build_workspace_bytes(T, E, R), dev)
    err = N.error_word(dev)
    N.check(lib.mkg_csr_build(head.data_ptr(), rel.data_ptr(), tail.data_ptr(), T, E, R, structs[0], structs[1],
                              ngroups.data_ptr(), ws.data_ptr(), ws.numel(), err.data_ptr(), N.stream_handle(dev)),
            "csr_build")
    g = ngroups.tolist()
    N.raise_device_errors(dev)
    res = []
    for o in outs:
        res += [o["row_ptr"], o["col_ind"], o["r_ind"], o["order"]]
    groups = []
    for o, G in zip(outs, g):
        groups += [o["row_group_ptr"], o["group_rel"][:G].clone(), o["group_edge_start"][:G].clone(),
                   o["group_edge_count"][:G].clone()]
    return tuple(res + groups)


def ind2ptr(index: torch.Tensor, size: int) -> torch.Tensor:
    """Row pointer of ``index`` (fastlog.cpp:9-16): int64 [size + 1]."""
    lib = N.load()
    N.require_cuda(index, "index")
    dev = index.device
    idx = index.to(torch.int64).contiguous()
    out = torch.empty(int(size) + 1, dtype=torch.int64, device=dev)
    ws = N.workspace(lib.mkg_ind2ptr_workspace_bytes(int(size)), dev)
    N.check(lib.mkg_ind2ptr(idx.data_ptr(), idx.numel(), int(size), out.data_ptr(), ws.data_ptr(), ws.numel(),
                            N.error_word(dev).data_ptr(), N.stream_handle(dev)), "ind2ptr")
    return out


class DeviceGraph:
    """A CSR pair resident on one GPU plus the fused engine's neighbour lists."""

    def __init__(self, csr, num_entities: int, num_relations: int):
        if len(csr) != 16:
            raise ValueError("expected the 16-tuple of build_csr_structure")
        dev = csr[0].device
        N.require_cuda(csr[0], "the CSR structure")
        self.device = dev
        self.csr = tuple(t.to(device=dev, dtype=dt).contiguous() for t, dt in zip(csr, CSR_DTYPES))
        self.num_entities = int(num_entities)
        self.num_relations = int(num_relations)
        self.num_facts = int(self.csr[1].numel())
        if int(self.csr[0].numel()) != self.num_entities + 1:
            raise ValueError(f"row_ptr has {self.csr[0].numel()} entries, expected E+1 = {self.num_entities + 1}")
        c = self.csr
        self.struct = N.Graph(
            self.num_entities, self.num_relations, self.num_facts,
            N.CsrDir(c[0].data_ptr(), c[1].data_ptr(), c[2].data_ptr(), c[3].data_ptr(), c[8].data_ptr(),
                     c[9].data_ptr(), c[10].data_ptr(), c[11].data_ptr(), c[9].numel()),
            N.CsrDir(c[4].data_ptr(), c[5].data_ptr(), c[6].data_ptr(), c[7].data_ptr(), c[12].data_ptr(),
                     c[13].data_ptr(), c[14].data_ptr(), c[15].data_ptr(), c[13].numel()))
        self._adj = None
        self._adj_keep = None
        self._facts = None
        self._cap = {}
        self.factor_writes = 0  # set_edge_factor calls so far (a caller can tell its factors are current)

    @classmethod
    def from_triples(cls, head: torch.Tensor, rel: torch.Tensor, tail: torch.Tensor, num_entities: int,
                     num_relations: int) -> "DeviceGraph":
        csr = build_csr_structure(head, tail, rel, num_entities, num_relations)
        return cls(csr, num_entities, num_relations)

    @classmethod
    def from_npy(cls, path, device: torch.device | str = "cuda", num_entities: int | None = None,
                 num_relations: int | None = None, chunk: int = 1 << 24) -> "DeviceGraph":
        """The graph of an ``N x 3`` (head, rel, tail) ``.npy`` fact file (the reference's
        ``load_facts(.., "npy")``, data.py:14-21, memory-mapped), streamed to the device in
        ``chunk``-row pieces through one pinned buffer, then built on the device.  Entity and
        relation counts default to max id + 1 (facts.py:19-23), taken on the device."""
        import numpy as np
        facts = np.load(path, mmap_mode="r")
        if facts.ndim != 2 or facts.shape[1] < 3:
            raise ValueError(f"expected an Nx3 fact array in {path}, got shape={facts.shape}")
        dev = torch.device(device)
        T = int(facts.shape[0])
        cols = [torch.empty(T, dtype=torch.int32, device=dev) for _ in range(3)]
        stage = torch.empty((min(chunk, max(T, 1)), 3), dtype=torch.int32, pin_memory=True)
        for a in range(0, T, chunk):
            b = min(T, a + chunk)
            piece = np.asarray(facts[a:b, :3])
            if piece.size and (piece.min() < 0 or piece.max() > np.iinfo(np.int32).max):
                raise ValueError("fact ids must lie in [0, 2^31)")
            stage[: b - a].copy_(torch.from_numpy(piece.astype(np.int32, copy=False)))
            dv = stage[: b - a].to(dev, non_blocking=True)
            for k in range(3):
                cols[k][a:b] = dv[:, k]
            torch.cuda.current_stream(dev).synchronize()  # the pinned buffer is reused
        head, rel, tail = cols
        if num_entities is None:
            num_entities = int(torch.maximum(head.max(), tail.max()).item()) + 1 if T else 1
        if num_relations is None:
            num_relations = int(rel.max().item()) + 1 if T else 1
        return cls.from_triples(head, rel, tail, int(num_entities), int(num_relations))

    # -------------------------------------------------------------- fused-engine lists
    def adjacency(self) -> N.Adjacency:
        if self._adj is None:
            lib = N.load()
            dev, E, T = self.device, self.num_entities, self.num_facts
            max_tasks = int(lib.mkg_adjacency_max_tasks(E, T))
            keep = dict(pull_ptr=torch.empty(E + 1, dtype=torch.int32, device=dev),
                        pull=torch.empty((2 * T, 4), dtype=torch.int32, device=dev),
                        push_ptr=torch.empty(E + 1, dtype=torch.int32, device=dev),
                        push=torch.empty((2 * T, 4), dtype=torch.int32, device=dev),
                        pull_tasks=torch.empty((max_tasks, 4), dtype=torch.int32, device=dev),
                        push_tasks=torch.empty((max_tasks, 4), dtype=torch.int32, device=dev))
            counts = torch.zeros(2, dtype=torch.int64, device=dev)
            adj = N.Adjacency(keep["pull_ptr"].data_ptr(), keep["pull"].data_ptr(), keep["push_ptr"].data_ptr(),
                              keep["push"].data_ptr(), keep["pull_tasks"].data_ptr(), 0,
                              keep["push_tasks"].data_ptr(), 0)
            ws = N.workspace(lib.mkg_adjacency_workspace_bytes(E), dev)
            N.check(lib.mkg_adjacency_build(C_ref(self.struct), adj, counts.data_ptr(), ws.data_ptr(), ws.numel(),
                                            N.error_word(dev).data_ptr(), N.stream_handle(dev)), "adjacency_build")
            n_pull, n_push = counts.tolist()
            N.raise_device_errors(dev)
            adj.num_pull_tasks = int(n_pull)
            adj.num_push_tasks = int(n_push)
            self._adj, self._adj_keep = adj, keep
        return self._adj

    def cap_index(self, cap: int) -> N.CapIndex:
        """The fused engine's edge-cap index for ``cap`` (0 .. MKG_DENSE_CAP_MAX): per-hop take
        tables are filled from it by the loop.  Built once per cap value and kept."""
        cap = int(cap)
        if cap not in self._cap:
            lib = N.load()
            dev, E, T = self.device, self.num_entities, self.num_facts
            adj = self.adjacency()
            ws = N.workspace(lib.mkg_cap_index_workspace_bytes(C_ref(self.struct)), dev)
            sizes = torch.zeros(2, dtype=torch.int64, device=dev)
            st = N.stream_handle(dev)
            N.check(lib.mkg_cap_index_sizes(C_ref(self.struct), cap, sizes.data_ptr(), ws.data_ptr(), ws.numel(), st),
                    "cap_index_sizes")
            n_slots, n_groups = (int(x) for x in sizes.tolist())
            keep = dict(slot_entity=torch.empty(max(n_slots, 1), dtype=torch.int32, device=dev),
                        slot_dir=torch.empty(max(n_slots, 1), dtype=torch.int32, device=dev),
                        slot_group=torch.empty(max(n_slots, 1), dtype=torch.int32, device=dev),
                        pull_cap=torch.empty((2 * T, 2), dtype=torch.int32, device=dev),
                        push_cap=torch.empty((2 * T, 2), dtype=torch.int32, device=dev),
                        capped_degree=torch.empty(max(E, 1), dtype=torch.int32, device=dev))
            ix = N.CapIndex(cap, n_slots, n_groups, *(keep[k].data_ptr() for k in
                                                       ("slot_entity", "slot_dir", "slot_group", "pull_cap",
                                                        "push_cap", "capped_degree")))
            N.check(lib.mkg_cap_index_build(C_ref(self.struct), C_ref(adj), C_ref(ix), ws.data_ptr(), ws.numel(),
                                            N.error_word(dev).data_ptr(), st), "cap_index_build")
            N.raise_device_errors(dev)
            self._cap[cap] = (ix, keep)
        return self._cap[cap][0]

    def push_degree(self) -> torch.Tensor:
        self.adjacency()
        p = self._adj_keep["push_ptr"]
        return (p[1:] - p[:-1]).to(torch.int64)

    def set_edge_factor(self, mask, weight, is_score: bool, scale: float, push_only: bool = False) -> None:
        """Writes the edge factor of every neighbour-list record; ``push_only`` leaves the pull
        list's factors as they were (the key-slab loop reads only the push list)."""
        lib = N.load()
        keep = []
        f = N.edge_factor(mask, weight, is_score, scale, keep)
        adj = self.adjacency()
        if push_only:
            adj = N.Adjacency(None, None, adj.push_ptr, adj.push, adj.pull_tasks, adj.num_pull_tasks,
                              adj.push_tasks, adj.num_push_tasks)
        N.check(lib.mkg_adjacency_set_factor(C_ref(self.struct), adj, C_ref(f), N.stream_handle(self.device)),
                "adjacency_set_factor")
        self.factor_writes += 1

    # -------------------------------------------------------------- per-fact endpoints
    def fact_table(self):
        if self._facts is None:
            lib = N.load()
            dev, T = self.device, self.num_facts
            h = torch.empty(T, dtype=torch.int32, device=dev)
            t = torch.empty(T, dtype=torch.int32, device=dev)
            r = torch.empty(T, dtype=torch.int16, device=dev)
            N.check(lib.mkg_fact_table(C_ref(self.struct), h.data_ptr(), t.data_ptr(), r.data_ptr(),
                                       N.error_word(dev).data_ptr(), N.stream_handle(dev)), "fact_table")
            self._facts = (h, t, r)
        return self._facts


def C_ref(obj):
    import ctypes
    return ctypes.byref(obj)


_CACHE: "OrderedDict[tuple, DeviceGraph]" = OrderedDict()
_CACHE_MAX = 4


def graph_from_csr(csr, num_entities: int, num_relations: int) -> DeviceGraph:
    """Cached ``DeviceGraph`` for a CSR tuple (keyed by tensor identity, as the reference
    caches its CSR by data pointers, proof.py:503-506).  The cache holds the tensors, so a
    key's memory cannot be reused by another graph while it is cached."""
    key = tuple((t.data_ptr(), t.numel(), t.dtype) for t in csr) + (int(num_entities), int(num_relations))
    g = _CACHE.get(key)
    if g is None:
        g = DeviceGraph(csr, num_entities, num_relations)
        g._source = tuple(csr)
        _CACHE[key] = g
        while len(_CACHE) > _CACHE_MAX:
            _CACHE.popitem(last=False)
    else:
        _CACHE.move_to_end(key)
    return g
