"""garfield_b200: the Garfield GMG query path on NVIDIA B200 (sm_100a).

Python host mirror of the C ABI declared in include/garfield.h.  The compute runs in
libgarfield_b200.so (hand-written CUDA); this module only marshals arrays.  Device
arrays are torch CUDA tensors (used as plain device memory); host arrays are numpy.

The reference (ZJU-DAILY/Garfield) exposes its query path as host functions inside one
CUDA translation unit; the mapping is:
  Index(...)                 real_dataset_test_multiD loading block (realdataset_search.cu:2118-2393)
  Index.plan(...)            intersection_area_mark_little_seg_V2 (real_dataset_adapter.cuh:390)
                             + get_partitions_access_order_V2 (gpu_graph.cu:11742)
  Index.search(...)          batch_graph_search_gpu_with_prefilter_and_postfilter (gpu_graph.cu:12464)
  Index.bruteforce(...)      naive_brute_force_with_filter (gpu_graph.cu:10782)
  read_* / write_*           loaders of tools.cuh / real_dataset_adapter.cuh (formats: Appendix of the docs)
If the shared library is missing the import still succeeds, but every call that needs
it raises: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

__all__ = [
    "GarfieldError", "lib", "lib_path", "SearchParams", "Index", "Plan", "NO_ID", "schedule_batches",
    "read_fvecs", "write_fvecs", "read_attrs", "write_attrs", "read_u32mat", "write_u32mat",
    "read_ranges", "write_ranges", "read_labels", "read_grid",
]

NO_ID = 0xFFFFFFFF
_PKG = Path(__file__).resolve().parent
lib_path = _PKG / "libgarfield_b200.so"


class GarfieldError(RuntimeError):
    def __init__(self, status: int, what: str, msg: str):
        super().__init__(f"{what}: status {status} ({msg})")
        self.status = status


class _IndexDesc(C.Structure):
    _fields_ = [
        ("n", C.c_uint32), ("dim", C.c_uint32), ("n_attr", C.c_uint32),
        ("vectors", C.c_void_p), ("attrs", C.c_void_p), ("grid", C.c_void_p),
        ("l_quant", C.c_void_p), ("r_quant", C.c_void_p), ("cell_of", C.c_void_p),
        ("degree", C.c_uint32), ("graphs", C.c_void_p), ("cross_e", C.c_uint32),
        ("cross", C.c_void_p), ("n_clusters", C.c_uint32), ("labels", C.c_void_p),
        ("f2h_factor", C.c_float), ("keep_fp32", C.c_uint32), ("host_graph", C.c_uint32),
        ("shard_cells", C.c_void_p), ("n_shard_cells", C.c_uint32),
        ("codec", C.c_uint32), ("codes", C.c_void_p), ("code_scales", C.c_void_p),
        ("code_zero_points", C.c_void_p), ("cross_spokesman", C.c_uint32),
    ]


class _IndexFiles(C.Structure):
    _fields_ = [
        ("data_path", C.c_char_p), ("cagra_prefix", C.c_char_p), ("cagra_suffix", C.c_char_p),
        ("global_graph", C.c_char_p), ("grid", C.c_char_p), ("attrs", C.c_char_p),
        ("cluster", C.c_char_p), ("degree", C.c_uint32), ("f2h_factor", C.c_float),
        ("keep_fp32", C.c_uint32), ("host_graph", C.c_uint32), ("codec", C.c_uint32),
        ("quantized", C.c_char_p), ("uniform_dims", C.c_uint32),
        ("uniform_shape", C.c_void_p),
        ("uniform_lo", C.c_float), ("uniform_hi", C.c_float),
    ]


class _SearchParams(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in
                ("L", "k", "width", "max_iter", "n_entry", "postfilter", "hash_slots", "test_wait", "exact_tc",
                 "route")]


class _BfParams(C.Structure):
    _fields_ = [("path", C.c_uint32), ("test_fallback_every", C.c_uint32), ("test_wait", C.c_uint32),
                ("stats_out", C.c_void_p)]


class _SearchStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("n_dist", "n_exp", "n_cross", "n_hops", "n_exact", "n_queries",
                                          "n_timeouts", "n_plan_fallbacks", "n_plan_reranked")]


class _IndexInfo(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in
                ("n", "dim", "n_attr", "n_cells", "degree", "cross_e", "n_clusters", "d_stored",
                 "min_cell_size", "cross_rows")] + [("device_bytes", C.c_uint64)]


_LIB = None
_P = C.c_void_p
_U32 = C.c_uint32
_PTR = C.POINTER


def lib() -> C.CDLL:
    """Load libgarfield_b200.so (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not lib_path.exists():
        raise GarfieldError(-1, "load", f"{lib_path} not built; run python -m garfield_b200.build")
    L = C.CDLL(str(lib_path))
    sig = {
        "gf_status_string": (C.c_char_p, [C.c_int]),
        "gf_last_error": (C.c_char_p, []),
        "gf_version": (C.c_char_p, []),
        "gf_search_defaults": (None, [_PTR(_SearchParams)]),
        "gf_index_create": (C.c_int, [_PTR(_IndexDesc), C.c_int, _PTR(_P)]),
        "gf_index_open": (C.c_int, [_PTR(_IndexFiles), C.c_int, _PTR(_P)]),
        "gf_index_info_get": (C.c_int, [_P, _PTR(_IndexInfo)]),
        "gf_index_entry_points": (C.c_int, [_P, _U32, _P]),
        "gf_index_destroy": (C.c_int, [_P]),
        "gf_plan_create": (C.c_int, [_P, _U32, _PTR(_P)]),
        "gf_plan_destroy": (C.c_int, [_P]),
        "gf_plan_queries": (C.c_int, [_P, _P, _P, _P, _P, _U32, C.c_float, _P]),
        "gf_plan_read": (C.c_int, [_P, _P, _P, _P, C.c_uint64, _P, _P]),
        "gf_search": (C.c_int, [_P, _P, _PTR(_SearchParams), _P, _P, _P]),
        "gf_search_stats_read": (C.c_int, [_P, _PTR(_SearchStats)]),
        "gf_search_host": (C.c_int, [_P, _P, _PTR(_SearchParams), _P, _P, _P, _U32, C.c_float, _P, _P, _P]),
        "gf_search_batched": (C.c_int, [_P, _P, _PTR(_SearchParams), _P, _P, _U32, _P, _P, _P]),
        "gf_search_keys": (C.c_int, [_P, _P, _PTR(_SearchParams), _P, _P]),
        "gf_merge_keys": (C.c_int, [_P, _P, _U32, _U32, _U32, _P, _P, _P]),
        "gf_schedule_batches": (C.c_int, [_P, _U32, _P, _P, _PTR(_U32), _PTR(C.c_uint64)]),
        "gf_schedule_batches_host": (C.c_int, [_U32, _U32, _P, _P, _P, _U32, _P, _P, _PTR(_U32),
                                               _PTR(C.c_uint64)]),
        "gf_bruteforce": (C.c_int, [_P, _P, _P, _P, _U32, _U32, _P, _P, _P]),
        "gf_bruteforce_ex": (C.c_int, [_P, _P, _P, _P, _U32, _U32, _P, _P, _PTR(_BfParams), _P]),
        "gf_index_assemble": (C.c_int, [_P, _U32]),
        "gf_search_fullgraph": (C.c_int, [_P, _P, _PTR(_SearchParams), _P, _P, _P]),
        "gf_free": (None, [_P]),
        "gf_read_fvecs": (C.c_int, [C.c_char_p, _PTR(_P), _PTR(_U32), _PTR(_U32)]),
        "gf_write_fvecs": (C.c_int, [C.c_char_p, _P, _U32, _U32]),
        "gf_read_u8bin": (C.c_int, [C.c_char_p, _PTR(_P), _PTR(_U32), _PTR(_U32)]),
        "gf_read_attrs": (C.c_int, [C.c_char_p, _PTR(_P), _PTR(_U32), _PTR(_U32)]),
        "gf_read_q": (C.c_int, [C.c_char_p, _PTR(_P), _PTR(_P), _PTR(_P), _PTR(_U32), _PTR(_U32)]),
        "gf_write_q": (C.c_int, [C.c_char_p, _P, _P, _P, _U32, _U32]),
        "gf_quantize_i8": (C.c_int, [_P, _U32, _U32, C.c_float, _P, _P, _P, _P]),
        "gf_quantize_i8_host": (C.c_int, [_P, _U32, _U32, C.c_float, _P, _P, _P]),
        "gf_write_attrs": (C.c_int, [C.c_char_p, _P, _U32, _U32]),
        "gf_read_u32mat": (C.c_int, [C.c_char_p, _PTR(_P), _PTR(_U32), _PTR(_U32)]),
        "gf_write_u32mat": (C.c_int, [C.c_char_p, _P, _U32, _U32]),
        "gf_read_ranges": (C.c_int, [C.c_char_p, _U32, _U32, _P, _P]),
        "gf_write_ranges": (C.c_int, [C.c_char_p, _P, _P, _U32, _U32]),
        "gf_read_labels": (C.c_int, [C.c_char_p, _PTR(_P), _PTR(_U32)]),
        "gf_read_grid": (C.c_int, [C.c_char_p, _PTR(_U32), _PTR(_U32), _PTR(_P), _PTR(_P), _PTR(_P), _PTR(_P)]),
        "gf_spokesman_host": (C.c_int, [_U32, _U32, _P, _U32, _P, _P, _P, _PTR(_U32)]),
        "gf_write_spokesman_graph": (C.c_int, [C.c_char_p, _U32, _U32, _U32, _P, _P, _P, _P]),
        "gf_read_spokesman_graph": (C.c_int, [C.c_char_p, _PTR(_U32), _PTR(_U32), _PTR(_U32), _PTR(_P), _PTR(_P),
                                              _PTR(_P), _PTR(_P)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _LIB = L
    return L


def _check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        raise GarfieldError(status, what, L.gf_last_error().decode(errors="replace"))


def _np_ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _dev_ptr(t):
    if t is None:
        return None
    import torch
    assert isinstance(t, torch.Tensor) and t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return C.c_void_p(t.data_ptr())


def _stream_ptr(stream):
    if stream is None:
        import torch
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)
    return C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


# ------------------------------------------------------------------ params

@dataclass
class SearchParams:
    """Search knobs; defaults are the reference's values (gpu_graph.cu:39, realdataset_search.cu:2495)."""
    L: int = 64
    k: int = 10
    width: int = 1
    max_iter: int = 10000
    n_entry: int = 0          # 0 = graph degree
    postfilter: int = 0xFFFFFFFF
    hash_slots: int = 0       # 0 = automatic
    test_wait: int = 0        # test hook: staging waits give up after this many polls and never complete
    exact_tc: int = 0         # 1: exact-route queries go to the tensor-core exact scan (fp32 rows)
    route: int = 0            # 1: also route by cost (box count vs cells x (L + 64)); needs exact_tc

    def _c(self) -> _SearchParams:
        return _SearchParams(self.L, self.k, self.width, self.max_iter, self.n_entry, self.postfilter,
                             self.hash_slots, self.test_wait, self.exact_tc, self.route)


# ------------------------------------------------------------------ index

class Index:
    """Device-resident GMG index (gf_index)."""

    def __init__(self, handle: C.c_void_p, keep: tuple = ()):
        self._h = handle
        self._keep = keep
        info = _IndexInfo()
        _check(lib().gf_index_info_get(self._h, C.byref(info)), "gf_index_info_get")
        self.n, self.dim, self.n_attr = info.n, info.dim, info.n_attr
        self.n_cells, self.degree, self.cross_e = info.n_cells, info.degree, info.cross_e
        self.n_clusters, self.min_cell_size = info.n_clusters, info.min_cell_size
        self.device_bytes = info.device_bytes
        self.cross_rows = info.cross_rows

    @classmethod
    def create(cls, *, vectors, attrs, grid, l_quant, r_quant, cell_of, graphs, degree, cross=None,
               cross_e=0, labels=None, f2h_factor=1.0, keep_fp32=True, host_graph=False, shard_cells=None,
               codec=0, codes=None, code_scales=None, code_zero_points=None, cross_spokesman=False,
               device=0) -> "Index":
        """Build from host arrays in the reference's layout (see gf_index_desc).  With
        host_graph the graphs and cross edges stay in pinned host memory (search with
        Plan.search_batched); with shard_cells the device holds only those cells (a shard
        of a cell-sharded index: Plan.search_keys + Index.merge_keys)."""
        vectors = np.ascontiguousarray(vectors, dtype=np.float32)
        attrs = np.ascontiguousarray(attrs, dtype=np.float32)
        grid = np.ascontiguousarray(grid, dtype=np.uint32)
        lq = np.ascontiguousarray(l_quant, dtype=np.float32)
        rq = np.ascontiguousarray(r_quant, dtype=np.float32)
        cell_of = np.ascontiguousarray(cell_of, dtype=np.uint32)
        graphs = np.ascontiguousarray(graphs, dtype=np.uint32)
        cross = None if cross is None else np.ascontiguousarray(cross, dtype=np.uint32)
        labels = None if labels is None else np.ascontiguousarray(labels, dtype=np.int32)
        n, dim = vectors.shape
        d = _IndexDesc()
        d.n, d.dim, d.n_attr = n, dim, attrs.shape[1]
        d.vectors, d.attrs, d.grid = _np_ptr(vectors), _np_ptr(attrs), _np_ptr(grid)
        d.l_quant, d.r_quant, d.cell_of = _np_ptr(lq), _np_ptr(rq), _np_ptr(cell_of)
        d.degree, d.graphs = degree, _np_ptr(graphs)
        d.cross_e, d.cross = (cross_e if cross is not None else 0), _np_ptr(cross)
        d.n_clusters, d.labels = (1 if labels is not None else 0), _np_ptr(labels)
        d.f2h_factor, d.keep_fp32 = f2h_factor, 1 if keep_fp32 else 0
        d.host_graph = 1 if host_graph else 0
        shard = None
        if shard_cells is not None:
            shard = np.ascontiguousarray(shard_cells, dtype=np.uint32)
            d.shard_cells, d.n_shard_cells = _np_ptr(shard), len(shard)
            d.keep_fp32 = 0
        d.codec = codec
        d.cross_spokesman = 1 if cross_spokesman else 0
        keep = []
        if codes is not None:
            codes = np.ascontiguousarray(codes).view(np.uint8)
            keep.append(codes)
            d.codes = _np_ptr(codes)
        if code_scales is not None:
            code_scales = np.ascontiguousarray(code_scales, dtype=np.float32)
            keep.append(code_scales)
            d.code_scales = _np_ptr(code_scales)
        if code_zero_points is not None:
            code_zero_points = np.ascontiguousarray(code_zero_points, dtype=np.int32)
            keep.append(code_zero_points)
            d.code_zero_points = _np_ptr(code_zero_points)
        h = C.c_void_p()
        _check(lib().gf_index_create(C.byref(d), device, C.byref(h)), "gf_index_create")
        return cls(h)

    @classmethod
    def open(cls, *, data_path, cagra_prefix, cagra_suffix, global_graph, grid=None, attrs, cluster=None,
             degree=32, f2h_factor=1.0, keep_fp32=False, device=0, uniform_shape=None, uniform_lo=0.0,
             uniform_hi=1e6, host_graph=False, codec=0, quantized=None) -> "Index":
        """Load the reference's index files (realdataset_search flags).  Without a grid file,
        `uniform_shape` gives the uniform grid of normaldataset_search."""
        f = _IndexFiles()
        f.data_path, f.cagra_prefix, f.cagra_suffix = (str(data_path).encode(), str(cagra_prefix).encode(),
                                                       str(cagra_suffix).encode())
        f.global_graph, f.attrs = str(global_graph).encode(), str(attrs).encode()
        f.grid = None if grid is None else str(grid).encode()
        f.cluster = None if cluster is None else str(cluster).encode()
        f.degree, f.f2h_factor, f.keep_fp32 = degree, f2h_factor, 1 if keep_fp32 else 0
        f.host_graph = 1 if host_graph else 0
        f.codec = codec
        f.quantized = None if quantized is None else str(quantized).encode()
        shape = None
        if uniform_shape is not None:
            shape = np.ascontiguousarray(uniform_shape, dtype=np.uint32)
            f.uniform_dims, f.uniform_shape = len(shape), _np_ptr(shape)
            f.uniform_lo, f.uniform_hi = uniform_lo, uniform_hi
        h = C.c_void_p()
        _check(lib().gf_index_open(C.byref(f), device, C.byref(h)), "gf_index_open")
        return cls(h)

    def close(self) -> None:
        if self._h:
            lib().gf_index_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def entry_points(self, n: int) -> np.ndarray:
        out = np.zeros(n, np.uint32)
        _check(lib().gf_index_entry_points(self._h, n, _np_ptr(out)), "gf_index_entry_points")
        return out

    def assemble(self, reserve: int = 2) -> None:
        """gf_index_assemble: the full-graph ablation's graph (assemble_edges) on the device."""
        _check(lib().gf_index_assemble(self._h, reserve), "gf_index_assemble")

    def plan(self, max_queries: int) -> "Plan":
        return Plan(self, max_queries)

    def merge_keys(self, keys, k: int, stream=None):
        """gf_merge_keys: keys (lists, qnum, k) int64 CUDA tensor -> (ids int32, dists)."""
        import torch
        lists, q = keys.shape[0], keys.shape[1]
        ids = torch.empty((q, k), dtype=torch.int32, device=keys.device)
        dist = torch.empty((q, k), dtype=torch.float32, device=keys.device)
        _check(lib().gf_merge_keys(self._h, _dev_ptr(keys), lists, q, k, _dev_ptr(ids), _dev_ptr(dist),
                                   _stream_ptr(stream)), "gf_merge_keys")
        return ids, dist

    def bruteforce(self, queries, lb, rb, k: int, stream=None, path: int = 0, test_fallback_every: int = 0,
                   stats=None, test_wait: int = 0):
        """Exact filtered k-NN on the device; returns (ids, dists) CUDA tensors.

        path: 0 automatic (tensor cores when available), 1 CUDA cores, 2 tensor cores.
        stats: optional int32 CUDA tensor of 3 words (queries answered by the CUDA-core
        kernel after the tensor-core pass, waits that ran out, 128 x 128 tile products)."""
        import torch
        q = queries.shape[0]
        ids = torch.empty((q, k), dtype=torch.int32, device=queries.device)
        dist = torch.empty((q, k), dtype=torch.float32, device=queries.device)
        if path == 0 and test_fallback_every == 0 and stats is None and test_wait == 0:
            _check(lib().gf_bruteforce(self._h, _dev_ptr(queries), _dev_ptr(lb), _dev_ptr(rb), q, k,
                                       _dev_ptr(ids), _dev_ptr(dist), _stream_ptr(stream)), "gf_bruteforce")
        else:
            prm = _BfParams(path, test_fallback_every, test_wait, _dev_ptr(stats).value if stats is not None else None)
            _check(lib().gf_bruteforce_ex(self._h, _dev_ptr(queries), _dev_ptr(lb), _dev_ptr(rb), q, k,
                                          _dev_ptr(ids), _dev_ptr(dist), C.byref(prm), _stream_ptr(stream)),
                   "gf_bruteforce_ex")
        return ids, dist

    def search(self, queries, lb, rb, params: SearchParams | None = None, prefilter: float = 0.0,
               plan: "Plan | None" = None, stream=None):
        """Plan + search on the device; returns (ids int32, dists) CUDA tensors (ids: global, NO_ID = -1)."""
        params = params or SearchParams()
        own = plan is None
        plan = plan or Plan(self, queries.shape[0])
        try:
            plan.build(queries, lb, rb, prefilter, stream)
            return plan.search(params, stream)
        finally:
            if own:
                plan.close()

    def search_host(self, queries: np.ndarray, lb: np.ndarray, rb: np.ndarray, plan: "Plan",
                    params: SearchParams | None = None, prefilter: float = 0.0, with_dist: bool = False,
                    stream=None):
        """End-to-end call from host memory (gf_search_host): H2D, plan, search, D2H."""
        params = params or SearchParams()
        q = queries.shape[0]
        ids = np.empty((q, params.k), np.uint32)
        dist = np.empty((q, params.k), np.float32) if with_dist else None
        cp = params._c()
        _check(lib().gf_search_host(self._h, plan._h, C.byref(cp), _np_ptr(queries), _np_ptr(lb), _np_ptr(rb),
                                    q, prefilter, _np_ptr(ids), _np_ptr(dist), _stream_ptr(stream)),
               "gf_search_host")
        return ids, dist


class Plan:
    """Planned query batch (gf_plan): cell lists in cluster-guided order."""

    def __init__(self, index: Index, max_queries: int):
        self.index = index
        self.max_queries = max_queries
        h = C.c_void_p()
        _check(lib().gf_plan_create(index._h, max_queries, C.byref(h)), "gf_plan_create")
        self._h = h
        self.qnum = 0

    def close(self) -> None:
        if self._h:
            lib().gf_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def build(self, queries, lb, rb, prefilter: float = 0.0, stream=None) -> None:
        self.qnum = queries.shape[0]
        _check(lib().gf_plan_queries(self.index._h, self._h, _dev_ptr(queries), _dev_ptr(lb), _dev_ptr(rb),
                                     self.qnum, prefilter, _stream_ptr(stream)), "gf_plan_queries")

    def read(self):
        """(counts, offsets, cells, top4, box_counts) as numpy (synchronises)."""
        q = self.qnum
        counts = np.zeros(q, np.uint32)
        offsets = np.zeros(q, np.uint32)
        top4 = np.zeros((q, 4), np.uint32)
        box = np.zeros(q, np.uint32)
        cap = q * max(self.index.n_cells, 1)
        cells = np.zeros(cap, np.uint32)
        _check(lib().gf_plan_read(self._h, _np_ptr(counts), _np_ptr(offsets), _np_ptr(cells), cap,
                                  _np_ptr(top4), _np_ptr(box)), "gf_plan_read")
        total = int(counts.sum())
        return counts, offsets, cells[:total], top4, box

    def search(self, params: SearchParams | None = None, stream=None, ids=None, dist=None):
        import torch
        params = params or SearchParams()
        dev = torch.device("cuda", torch.cuda.current_device())
        if ids is None:
            ids = torch.empty((self.qnum, params.k), dtype=torch.int32, device=dev)
        if dist is None:
            dist = torch.empty((self.qnum, params.k), dtype=torch.float32, device=dev)
        cp = params._c()
        _check(lib().gf_search(self.index._h, self._h, C.byref(cp), _dev_ptr(ids), _dev_ptr(dist),
                               _stream_ptr(stream)), "gf_search")
        return ids, dist

    def search_fullgraph(self, params: SearchParams | None = None, stream=None, ids=None, dist=None):
        """gf_search_fullgraph: the full-graph post-filter ablation over the index's assembled
        graph (Index.assemble first)."""
        import torch
        params = params or SearchParams()
        dev = torch.device("cuda", torch.cuda.current_device())
        if ids is None:
            ids = torch.empty((self.qnum, params.k), dtype=torch.int32, device=dev)
        if dist is None:
            dist = torch.empty((self.qnum, params.k), dtype=torch.float32, device=dev)
        cp = params._c()
        _check(lib().gf_search_fullgraph(self.index._h, self._h, C.byref(cp), _dev_ptr(ids), _dev_ptr(dist),
                                         _stream_ptr(stream)), "gf_search_fullgraph")
        return ids, dist

    def search_batched(self, batches, params: SearchParams | None = None, stream=None, ids=None, dist=None):
        """gf_search_batched: `batches` is a list of cell-id lists (each cell in at most one)."""
        import torch
        params = params or SearchParams()
        dev = torch.device("cuda", torch.cuda.current_device())
        if ids is None:
            ids = torch.empty((self.qnum, params.k), dtype=torch.int32, device=dev)
        if dist is None:
            dist = torch.empty((self.qnum, params.k), dtype=torch.float32, device=dev)
        sizes = np.array([len(b) for b in batches], np.uint32)
        cells = np.ascontiguousarray(np.concatenate([np.asarray(b, np.uint32) for b in batches])
                                     if len(batches) else np.zeros(0, np.uint32), dtype=np.uint32)
        cp = params._c()
        _check(lib().gf_search_batched(self.index._h, self._h, C.byref(cp), _np_ptr(cells), _np_ptr(sizes),
                                       len(batches), _dev_ptr(ids), _dev_ptr(dist), _stream_ptr(stream)),
               "gf_search_batched")
        return ids, dist

    def search_keys(self, params: SearchParams | None = None, stream=None, keys=None):
        """gf_search_keys: (qnum, k) int64 CUDA tensor of merge keys."""
        import torch
        params = params or SearchParams()
        if keys is None:
            keys = torch.empty((self.qnum, params.k), dtype=torch.int64,
                               device=torch.device("cuda", torch.cuda.current_device()))
        cp = params._c()
        _check(lib().gf_search_keys(self.index._h, self._h, C.byref(cp), _dev_ptr(keys), _stream_ptr(stream)),
               "gf_search_keys")
        return keys

    def schedule(self, max_cells: int):
        """gf_schedule_batches: (list of cell lists, splits) for search_batched."""
        n = self.index.n_cells
        cells, sizes = np.zeros(n, np.uint32), np.zeros(n, np.uint32)
        nb, splits = _U32(), C.c_uint64()
        _check(lib().gf_schedule_batches(self._h, max_cells, _np_ptr(cells), _np_ptr(sizes), C.byref(nb),
                                         C.byref(splits)), "gf_schedule_batches")
        return _unpack_batches(cells, sizes, nb.value), int(splits.value)

    def stats(self) -> dict:
        s = _SearchStats()
        _check(lib().gf_search_stats_read(self._h, C.byref(s)), "gf_search_stats_read")
        return {n: getattr(s, n) for n, _ in _SearchStats._fields_}


# ------------------------------------------------------------------ file formats

def _unpack_batches(cells, sizes, nb):
    out, o = [], 0
    for b in range(nb):
        out.append(cells[o:o + int(sizes[b])].tolist())
        o += int(sizes[b])
    return out


def schedule_batches(ncells: int, counts, offsets, cells, max_cells: int):
    """gf_schedule_batches_host on host plan arrays: (list of cell lists, splits)."""
    counts = np.ascontiguousarray(counts, np.uint32)
    offsets = np.ascontiguousarray(offsets, np.uint32)
    cells = np.ascontiguousarray(cells, np.uint32)
    bc, bs = np.zeros(max(ncells, 1), np.uint32), np.zeros(max(ncells, 1), np.uint32)
    nb, splits = _U32(), C.c_uint64()
    _check(lib().gf_schedule_batches_host(ncells, len(counts), _np_ptr(counts), _np_ptr(offsets), _np_ptr(cells),
                                          max_cells, _np_ptr(bc), _np_ptr(bs), C.byref(nb), C.byref(splits)),
           "gf_schedule_batches_host")
    return _unpack_batches(bc, bs, nb.value), int(splits.value)


def quantize_i8_host(data: np.ndarray, alpha: float = 1.0):
    """gf_quantize_i8_host: (codes int8 n x dim, scales, zero points)."""
    data = np.ascontiguousarray(data, dtype=np.float32)
    n, dim = data.shape
    q = np.zeros((n, dim), np.int8)
    sc, zp = np.zeros(dim, np.float32), np.zeros(dim, np.int32)
    _check(lib().gf_quantize_i8_host(_np_ptr(data), n, dim, alpha, _np_ptr(q), _np_ptr(sc), _np_ptr(zp)),
           "gf_quantize_i8_host")
    return q, sc, zp


def quantize_i8(data, alpha: float = 1.0, stream=None):
    """gf_quantize_i8 on a CUDA tensor: (codes int8, scales, zero points) CUDA tensors."""
    import torch
    n, dim = data.shape
    q = torch.empty((n, dim), dtype=torch.int8, device=data.device)
    sc = torch.empty(dim, dtype=torch.float32, device=data.device)
    zp = torch.empty(dim, dtype=torch.int32, device=data.device)
    _check(lib().gf_quantize_i8(_dev_ptr(data), n, dim, alpha, _dev_ptr(q), _dev_ptr(sc), _dev_ptr(zp),
                                _stream_ptr(stream)), "gf_quantize_i8")
    return q, sc, zp


def read_q(path):
    """.q file -> (codes int8 n x dim, scales, zero points)."""
    q, sc, zp = _P(), _P(), _P()
    n, d = _U32(), _U32()
    _check(lib().gf_read_q(str(path).encode(), C.byref(q), C.byref(sc), C.byref(zp), C.byref(n), C.byref(d)),
           "gf_read_q")
    codes = _take(q, n.value * d.value, np.int8).reshape(n.value, d.value)
    return codes, _take(sc, d.value, np.float32), _take(zp, d.value, np.int32)


def write_q(path, codes, scales, zero_points) -> None:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    sc = np.ascontiguousarray(scales, dtype=np.float32)
    zp = np.ascontiguousarray(zero_points, dtype=np.int32)
    _check(lib().gf_write_q(str(path).encode(), _np_ptr(codes), _np_ptr(sc), _np_ptr(zp), codes.shape[0],
                            codes.shape[1]), "gf_write_q")


def _take(ptr: C.c_void_p, count: int, dtype) -> np.ndarray:
    arr = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(np.ctypeslib.as_ctypes_type(dtype))), shape=(count,)).copy()
    lib().gf_free(ptr)
    return arr


def read_fvecs(path) -> np.ndarray:
    p, n, d = C.c_void_p(), C.c_uint32(), C.c_uint32()
    _check(lib().gf_read_fvecs(str(path).encode(), C.byref(p), C.byref(n), C.byref(d)), "gf_read_fvecs")
    return _take(p, n.value * d.value, np.float32).reshape(n.value, d.value)


def write_fvecs(path, data: np.ndarray) -> None:
    a = np.ascontiguousarray(data, np.float32)
    _check(lib().gf_write_fvecs(str(path).encode(), _np_ptr(a), a.shape[0], a.shape[1]), "gf_write_fvecs")


def read_attrs(path) -> np.ndarray:
    p, n, a = C.c_void_p(), C.c_uint32(), C.c_uint32()
    _check(lib().gf_read_attrs(str(path).encode(), C.byref(p), C.byref(n), C.byref(a)), "gf_read_attrs")
    return _take(p, n.value * a.value, np.int32).reshape(n.value, a.value)


def write_attrs(path, attrs: np.ndarray) -> None:
    a = np.ascontiguousarray(attrs, np.int32)
    _check(lib().gf_write_attrs(str(path).encode(), _np_ptr(a), a.shape[0], a.shape[1]), "gf_write_attrs")


def read_u32mat(path) -> np.ndarray:
    p, n, k = C.c_void_p(), C.c_uint32(), C.c_uint32()
    _check(lib().gf_read_u32mat(str(path).encode(), C.byref(p), C.byref(n), C.byref(k)), "gf_read_u32mat")
    return _take(p, n.value * k.value, np.uint32).reshape(n.value, k.value)


def write_u32mat(path, m: np.ndarray) -> None:
    a = np.ascontiguousarray(m, np.uint32)
    _check(lib().gf_write_u32mat(str(path).encode(), _np_ptr(a), a.shape[0], a.shape[1]), "gf_write_u32mat")


def read_ranges(path, qnum: int, a: int):
    lo = np.zeros((qnum, a), np.int32)
    hi = np.zeros((qnum, a), np.int32)
    _check(lib().gf_read_ranges(str(path).encode(), qnum, a, _np_ptr(lo), _np_ptr(hi)), "gf_read_ranges")
    return lo, hi


def write_ranges(path, lo: np.ndarray, hi: np.ndarray) -> None:
    lo = np.ascontiguousarray(lo, np.int32)
    hi = np.ascontiguousarray(hi, np.int32)
    _check(lib().gf_write_ranges(str(path).encode(), _np_ptr(lo), _np_ptr(hi), lo.shape[0], lo.shape[1]),
           "gf_write_ranges")


def read_labels(path) -> np.ndarray:
    p, n = C.c_void_p(), C.c_uint32()
    _check(lib().gf_read_labels(str(path).encode(), C.byref(p), C.byref(n)), "gf_read_labels")
    return _take(p, n.value, np.int32)


def read_grid(path):
    """(grid, l_quant, r_quant, cell_of) of a grid_info file."""
    n, a = C.c_uint32(), C.c_uint32()
    g, lq, rq, co = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
    _check(lib().gf_read_grid(str(path).encode(), C.byref(n), C.byref(a), C.byref(g), C.byref(lq), C.byref(rq),
                              C.byref(co)), "gf_read_grid")
    grid = _take(g, a.value, np.uint32)
    tot = int(grid.sum())
    return grid, _take(lq, tot, np.int32), _take(rq, tot, np.int32), _take(co, n.value, np.uint32)


def spokesman(cell_sizes, graphs):
    """gf_spokesman_host: (spokesman position, spokesman rank, number of spokesmen) of every
    position (cell order) from the per-cell graphs (n x R local ids, rows in cell order)."""
    sizes = np.ascontiguousarray(cell_sizes, np.uint32)
    g = np.ascontiguousarray(graphs, np.uint32)
    n = g.shape[0]
    spk = np.zeros(n, np.uint32)
    rank = np.zeros(n, np.uint32)
    ns = C.c_uint32()
    _check(lib().gf_spokesman_host(n, len(sizes), _np_ptr(sizes), g.shape[1], _np_ptr(g), _np_ptr(spk), _np_ptr(rank),
                                   C.byref(ns)), "gf_spokesman_host")
    return spk, rank, ns.value


def compress_cross(cell_of, graphs, cross, cross_e: int):
    """The reference's compressed cross graph (compress_global_graph_extreme, tools.cuh:917-1010)
    from index arrays in the reference layout (global order): returns (center_num, col_offset,
    center_pos, edges) with center_pos indexed by position (cell order) and edges
    n_cells x n_spokesmen x E local ids, as gf_write_spokesman_graph writes them."""
    cell_of = np.asarray(cell_of, np.uint32)
    P = int(cell_of.max()) + 1
    order = np.argsort(cell_of, kind="stable")                    # position -> global id
    sizes = np.bincount(cell_of, minlength=P).astype(np.uint32)
    spk, rank, ns = spokesman(sizes, np.asarray(graphs, np.uint32))
    heads = np.nonzero(spk == np.arange(len(spk)))[0]              # spokesman positions, rank order
    seg = np.concatenate([[0], np.cumsum(sizes)])
    center_num = np.array([((heads >= seg[c]) & (heads < seg[c + 1])).sum() for c in range(P)], np.uint32)
    col_offset = np.concatenate([[0], np.cumsum(center_num)[:-1]]).astype(np.uint32)
    x = np.asarray(cross, np.uint32).reshape(len(cell_of), P, cross_e)[order[heads]]  # ns x P x E
    edges = np.ascontiguousarray(x.transpose(1, 0, 2))
    return center_num, col_offset, rank.astype(np.uint32), edges


def write_spokesman_graph(path, center_num, col_offset, center_pos, edges) -> None:
    cn = np.ascontiguousarray(center_num, np.uint32)
    co = np.ascontiguousarray(col_offset, np.uint32)
    cp = np.ascontiguousarray(center_pos, np.uint32)
    e = np.ascontiguousarray(edges, np.uint32)
    _check(lib().gf_write_spokesman_graph(str(path).encode(), len(cp), len(cn), e.shape[2], _np_ptr(cn), _np_ptr(co),
                                          _np_ptr(cp), _np_ptr(e)), "gf_write_spokesman_graph")


def read_spokesman_graph(path):
    n, P, E = C.c_uint32(), C.c_uint32(), C.c_uint32()
    a, b, c, d = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
    _check(lib().gf_read_spokesman_graph(str(path).encode(), C.byref(n), C.byref(P), C.byref(E), C.byref(a),
                                         C.byref(b), C.byref(c), C.byref(d)), "gf_read_spokesman_graph")
    cn = _take(a, P.value, np.uint32)
    total = int(cn.sum())
    return (cn, _take(b, P.value, np.uint32), _take(c, n.value, np.uint32),
            _take(d, P.value * total * E.value, np.uint32).reshape(P.value, total, E.value))


def recall(res: np.ndarray, gt: np.ndarray) -> float:
    """Mean over queries of |res ∩ gt| / |gt| (cal_recall_show_partition_multi_attrs,
    tools.cuh:456-544); an empty ground-truth row counts as 1; NO_ID entries are ignored."""
    res = np.asarray(res, np.uint32)
    gt = np.asarray(gt, np.uint32)
    total = 0.0
    for r, g in zip(res, gt):
        g = g[g != NO_ID]
        total += 1.0 if g.size == 0 else np.isin(g, r[r != NO_ID]).sum() / g.size
    return total / max(1, res.shape[0])


def version() -> str:
    return lib().gf_version().decode()


if os.environ.get("GARFIELD_B200_EAGER_LOAD"):
    lib()
