"""ctypes binding of the CPU oracle (gf_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline as the checker.  No product code path imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
EMPTY = 0xFFFFFFFF


def build() -> Path:
    src = HERE / "gf_oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        env = dict(os.environ)
        env.pop("CC", None)
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return LIB


_L = None


class OrcIndex(C.Structure):
    _fields_ = [("n", C.c_uint32), ("d8", C.c_uint32), ("a", C.c_uint32), ("ncells", C.c_uint32),
                ("degree", C.c_uint32), ("cross_e", C.c_uint32), ("vec16", C.c_void_p), ("attrs", C.c_void_p),
                ("cell_of", C.c_void_p), ("graphs", C.c_void_p), ("cross", C.c_void_p),
                ("codec", C.c_uint32), ("d16", C.c_uint32), ("vec8", C.c_void_p), ("scale", C.c_void_p),
                ("bias", C.c_void_p)]


class OrcParams(C.Structure):
    _fields_ = [("L", C.c_uint32), ("K", C.c_uint32), ("width", C.c_uint32), ("max_iter", C.c_uint32),
                ("postfilter", C.c_uint32), ("prefilter", C.c_float), ("n_entry", C.c_uint32)]


def lib() -> C.CDLL:
    global _L
    if _L is None:
        build()
        _L = C.CDLL(str(LIB))
        P, U = C.c_void_p, C.c_uint32
        _L.orc_dist16.restype = C.c_float
        _L.orc_dist16.argtypes = [P, P, U]
        _L.orc_dist32.restype = C.c_float
        _L.orc_dist32.argtypes = [P, P, U]
        _L.orc_dist8.restype = C.c_float
        _L.orc_dist8.argtypes = [P, P, P, P, U, U]
        _L.orc_quantize_i8.argtypes = [P, U, U, C.c_float, P, P, P]
        _L.orc_spokesman.argtypes = [P, U, P, U, P, P]
        _L.orc_spokesman.restype = U
        _L.orc_dist_seq.restype = C.c_float
        _L.orc_dist_seq.argtypes = [P, P, U]
        _L.orc_f2h.argtypes = [P, U, U, U, C.c_float, P]
        _L.orc_count_in_box.argtypes = [P, U, U, P, P, U, P]
        _L.orc_bruteforce.argtypes = [P, U, U, P, U, P, P, P, U, U, P, P, C.c_int]
        _L.orc_plan_cells.restype = C.c_long
        _L.orc_plan_cells.argtypes = [P, P, U, U, P, P, P, P, P, P, C.c_uint64]
        _L.orc_cluster_info.argtypes = [P, U, U, P, P, U, U, P, P]
        _L.orc_order_cells.argtypes = [P, U, U, P, U, P, P, P, P, P]
        _L.orc_search.argtypes = [C.POINTER(OrcIndex), C.POINTER(OrcParams), P, U, C.c_float, P, P, U, P, P, P, P,
                                  P, P, P, P, C.c_int]
        _L.orc_search_batched.argtypes = [C.POINTER(OrcIndex), C.POINTER(OrcParams), P, U, C.c_float, P, P, U, P,
                                          P, P, P, P, P, U, P, P, P, C.c_int]
        _L.orc_assemble.argtypes = [C.POINTER(OrcIndex), U, P]
        _L.orc_search_fullgraph.argtypes = [C.POINTER(OrcIndex), C.POINTER(OrcParams), P, U, P, U, C.c_float, P, P,
                                            U, P, P, P, P, C.c_int]
        _L.orc_recall.restype = C.c_double
        _L.orc_recall.argtypes = [P, U, P, U, U]
    return _L


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def f2h(x: np.ndarray, d_pad: int, alpha: float = 1.0) -> np.ndarray:
    x = _c(x, np.float32)
    n, dim = x.shape
    out = np.zeros((n, d_pad), np.uint16)
    lib().orc_f2h(_p(x), n, dim, d_pad, alpha, _p(out))
    return out


def pad(x: np.ndarray, mult: int) -> np.ndarray:
    n, d = x.shape
    dp = (d + mult - 1) // mult * mult
    out = np.zeros((n, dp), np.float32)
    out[:, :d] = x
    return out


def dist16(q16: np.ndarray, x16: np.ndarray) -> float:
    q16, x16 = _c(q16, np.uint16), _c(x16, np.uint16)
    return lib().orc_dist16(_p(q16), _p(x16), q16.shape[-1])


def dist32(q: np.ndarray, x: np.ndarray) -> float:
    q, x = _c(q, np.float32), _c(x, np.float32)
    return lib().orc_dist32(_p(q), _p(x), q.shape[-1])


def bruteforce(data, attrs, queries, lo, hi, k: int, threads: int = 0):
    """Exact filtered top-k: (ids uint32 q x k, squared dists)."""
    d4 = pad(data, 4)
    q4 = pad(queries, 4)
    attrs = _c(attrs, np.float32)
    lo, hi = _c(lo, np.float32), _c(hi, np.float32)
    qn = q4.shape[0]
    ids = np.zeros((qn, k), np.uint32)
    dist = np.zeros((qn, k), np.float32)
    lib().orc_bruteforce(_p(d4), d4.shape[0], d4.shape[1], _p(attrs), attrs.shape[1], _p(q4), _p(lo), _p(hi),
                         qn, k, _p(ids), _p(dist), threads)
    return ids, dist


def count_in_box(attrs, lo, hi):
    attrs, lo, hi = _c(attrs, np.float32), _c(lo, np.float32), _c(hi, np.float32)
    out = np.zeros(lo.shape[0], np.uint32)
    lib().orc_count_in_box(_p(attrs), attrs.shape[0], attrs.shape[1], _p(lo), _p(hi), lo.shape[0], _p(out))
    return out


def plan_cells(lo, hi, grid, l_quant, r_quant):
    lo, hi = _c(lo, np.float32), _c(hi, np.float32)
    grid = _c(grid, np.uint32)
    lq, rq = _c(l_quant, np.float32), _c(r_quant, np.float32)
    qn, a = lo.shape
    counts = np.zeros(qn, np.uint32)
    offsets = np.zeros(qn, np.uint32)
    cap = qn * int(np.prod(grid)) + 1
    cells = np.zeros(cap, np.uint32)
    tot = lib().orc_plan_cells(_p(lo), _p(hi), qn, a, _p(grid), _p(lq), _p(rq), _p(counts), _p(offsets), _p(cells),
                               cap)
    assert tot >= 0
    return counts, offsets, cells[:tot].copy()


def cluster_info(data, labels, cell_of, ncells: int):
    data = _c(data, np.float32)
    labels = _c(labels, np.int32)
    cell_of = _c(cell_of, np.uint32)
    C_ = int(labels.max()) + 1
    cent = np.zeros((C_, data.shape[1]), np.float32)
    hist = np.zeros((ncells, C_), np.uint32)
    lib().orc_cluster_info(_p(data), data.shape[0], data.shape[1], _p(labels), _p(cell_of), ncells, C_, _p(cent),
                           _p(hist))
    return cent, hist


def order_cells(queries, centroids, hist, counts, offsets, cells):
    queries, centroids = _c(queries, np.float32), _c(centroids, np.float32)
    hist = _c(hist, np.uint32)
    counts, offsets = _c(counts, np.uint32), _c(offsets, np.uint32)
    cells = _c(cells, np.uint32).copy()
    top4 = np.zeros((queries.shape[0], 4), np.uint32)
    lib().orc_order_cells(_p(queries), queries.shape[0], queries.shape[1], _p(centroids), centroids.shape[0],
                          _p(hist), _p(counts), _p(offsets), _p(cells), _p(top4))
    return cells, top4


def spokesman(sizes, graphs):
    """tools.cuh:917-935 (compress_global_graph_extreme): (spokesman position, rank, count)
    of every position; graphs are n x R local ids with rows in position (cell) order."""
    sizes = np.ascontiguousarray(sizes, np.uint32)
    g = np.ascontiguousarray(graphs, np.uint32)
    spk = np.zeros(g.shape[0], np.uint32)
    rank = np.zeros(g.shape[0], np.uint32)
    ns = lib().orc_spokesman(_p(sizes), len(sizes), _p(g), g.shape[1], _p(spk), _p(rank))
    return spk, rank, int(ns)


def expand_spokesman_cross(cell_of, graphs, cross):
    """Cross edges as a spokesman-compressed index uses them, in the reference layout
    (global order): the row of every point is replaced by its spokesman's row."""
    cell_of = np.asarray(cell_of, np.uint32)
    order = np.argsort(cell_of, kind="stable")  # position -> global id
    sizes = np.bincount(cell_of, minlength=int(cell_of.max()) + 1)
    spk, _, _ = spokesman(sizes, np.asarray(graphs, np.uint32))
    out = np.empty_like(np.asarray(cross))
    out[order] = np.asarray(cross)[order[spk]]
    return out


def quantize_i8(data, alpha: float = 1.0):
    """orc_quantize_i8: (q int8 n x dim, scales fp32 dim, zero_points int32 dim)."""
    data = _c(data, np.float32)
    n, dim = data.shape
    q = np.zeros((n, dim), np.int8)
    sc = np.zeros(dim, np.float32)
    zp = np.zeros(dim, np.int32)
    lib().orc_quantize_i8(_p(data), n, dim, alpha, _p(q), _p(sc), _p(zp))
    return q, sc, zp


def byte_rows(q, scales, zero_points, codec: int):
    """Byte rows padded to a multiple of 16 with per-element scale and bias (orc_dist8);
    codec 1 = int8 (bias = zero_point + 128), 2 = uint8 (bias = zero_point)."""
    q = np.ascontiguousarray(q)
    n, dim = q.shape
    d16 = (dim + 15) // 16 * 16
    rows = np.zeros((n, d16), np.uint8)
    rows[:, :dim] = q.view(np.uint8)
    sc = np.zeros(d16, np.float32)
    bias = np.zeros(d16, np.float32)
    sc[:dim] = scales
    bias[:dim] = np.asarray(zero_points, np.float32) + (128.0 if codec == 1 else 0.0)
    return rows, sc, bias, d16


def dist8(q, row, scale, bias, codec: int) -> float:
    return lib().orc_dist8(_p(_c(q, np.float32)), _p(_c(row, np.uint8)), _p(_c(scale, np.float32)),
                           _p(_c(bias, np.float32)), 0x80 if codec == 1 else 0, len(row))


def search(index_arrays, vectors, attrs, queries, lo, hi, counts, offsets, cells, entry, *, L, K, width=1,
           max_iter=10000, postfilter=0xFFFFFFFF, prefilter=0.0, box_counts=None, alpha=1.0, threads=0,
           batches=None, codec=0, codes=None, scales=None, zero_points=None):
    """Beam search restatement; index_arrays: an indexbuild.GmgArrays (reference layout).

    With `batches` (a list of cell lists), the batched driver orc_search_batched runs
    instead: each batch is searched on its own and the results merged.  codec 1 / 2:
    distances to int8 / uint8 rows `codes` (n x dim, global order) with per-dimension
    `scales` and `zero_points` (orc_dist8) instead of fp16 rows."""
    vectors = _c(vectors, np.float32)
    n, dim = vectors.shape
    d8 = (dim + 7) // 8 * 8
    vec16 = f2h(vectors, d8, alpha)
    attrs = _c(attrs, np.float32)
    cell_of = _c(index_arrays.cell_of, np.uint32)
    graphs = _c(index_arrays.graphs, np.uint32)
    cross = _c(index_arrays.cross, np.uint32)
    ncells = int(np.prod(index_arrays.grid))
    ix = OrcIndex(n, d8, attrs.shape[1], ncells, index_arrays.degree, index_arrays.cross_e,
                  _p(vec16), _p(attrs), _p(cell_of), _p(graphs), _p(cross))
    if codec:
        rows, sc8, bias8, d16 = byte_rows(codes, scales, zero_points, codec)
        ix.codec, ix.d16, ix.vec8, ix.scale, ix.bias = codec, d16, _p(rows), _p(sc8), _p(bias8)
    entry = _c(entry, np.uint32)
    prm = OrcParams(L, K, width, max_iter, postfilter, prefilter, len(entry))
    queries = _c(queries, np.float32)
    lo, hi = _c(lo, np.float32), _c(hi, np.float32)
    counts, offsets, cells = _c(counts, np.uint32), _c(offsets, np.uint32), _c(cells, np.uint32)
    box = None if box_counts is None else _c(box_counts, np.uint32)
    qn = queries.shape[0]
    ids = np.zeros((qn, K), np.uint32)
    dist = np.zeros((qn, K), np.float32)
    stats = np.zeros(4, np.uint64)
    if batches is None:
        lib().orc_search(C.byref(ix), C.byref(prm), _p(queries), dim, alpha, _p(lo), _p(hi), qn, _p(counts),
                         _p(offsets), _p(cells), _p(box), _p(entry), _p(ids), _p(dist), _p(stats), threads)
    else:
        batch_of = np.full(ncells, 0xFFFFFFFF, np.uint32)
        for b, cl in enumerate(batches):
            for c in cl:
                batch_of[int(c)] = b
        lib().orc_search_batched(C.byref(ix), C.byref(prm), _p(queries), dim, alpha, _p(lo), _p(hi), qn,
                                 _p(counts), _p(offsets), _p(cells), _p(box), _p(entry), _p(batch_of), len(batches),
                                 _p(ids), _p(dist), _p(stats), threads)
    return ids, dist, stats


def _orc_index(index_arrays, vectors, attrs, alpha):
    vectors = _c(vectors, np.float32)
    n, dim = vectors.shape
    d8 = (dim + 7) // 8 * 8
    keep = dict(vec16=f2h(vectors, d8, alpha), attrs=_c(attrs, np.float32),
                cell_of=_c(index_arrays.cell_of, np.uint32), graphs=_c(index_arrays.graphs, np.uint32),
                cross=_c(index_arrays.cross, np.uint32))
    ix = OrcIndex(n, d8, keep["attrs"].shape[1], int(np.prod(index_arrays.grid)), index_arrays.degree,
                  index_arrays.cross_e, _p(keep["vec16"]), _p(keep["attrs"]), _p(keep["cell_of"]),
                  _p(keep["graphs"]), _p(keep["cross"]))
    return ix, keep


def assemble(index_arrays, reserve: int = 2):
    """full_graph_search.cuh:984-997 (assemble_edges): the full-graph ablation's graph,
    n x (cells * reserve) positions, rows in position order."""
    n = len(index_arrays.cell_of)
    zeros = np.zeros((n, 1), np.float32)
    ix, keep = _orc_index(index_arrays, zeros, np.zeros((n, 1), np.float32), 1.0)
    out = np.zeros((n, ix.ncells * reserve), np.uint32)
    lib().orc_assemble(C.byref(ix), reserve, _p(out))
    return out


def search_fullgraph(index_arrays, vectors, attrs, queries, lo, hi, entry_pos, *, L, K, width=1, reserve=2,
                     max_iter=10000, alpha=1.0, threads=0):
    """full_graph_search_postfiltering (full_graph_search.cuh:179-593) over assemble()'s
    graph of the whole index, box applied at the end; entry_pos are positions."""
    ix, keep = _orc_index(index_arrays, vectors, attrs, alpha)
    fg = assemble(index_arrays, reserve)
    entry = _c(entry_pos, np.uint32)
    prm = OrcParams(L, K, width, max_iter, 0xFFFFFFFF, 0.0, len(entry))
    queries = _c(queries, np.float32)
    lo, hi = _c(lo, np.float32), _c(hi, np.float32)
    qn, dim = queries.shape
    ids = np.zeros((qn, K), np.uint32)
    dist = np.zeros((qn, K), np.float32)
    stats = np.zeros(4, np.uint64)
    lib().orc_search_fullgraph(C.byref(ix), C.byref(prm), _p(fg), fg.shape[1], _p(queries), dim, alpha, _p(lo),
                               _p(hi), qn, _p(entry), _p(ids), _p(dist), _p(stats), threads)
    return ids, dist, stats


def recall(res, gt) -> float:
    res, gt = _c(res, np.uint32), _c(gt, np.uint32)
    return lib().orc_recall(_p(res), res.shape[1], _p(gt), gt.shape[1], res.shape[0])
