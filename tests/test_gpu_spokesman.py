"""Search on a spokesman-compressed index (gf_index_desc.cross_spokesman; the cross-edge
compression of compress_global_graph_extreme, tools.cuh:917-1010) against the oracle's
search over the expanded cross edges (each point's row replaced by its spokesman's row):
ids and canonical distances bit for bit, for whole-index and batched searches (rows
device-resident or streamed from pinned host memory); recall beside the uncompressed index."""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def make(c, spokesman):
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                           cross_spokesman=spokesman)


@pytest.mark.parametrize("which", ["small", "odd"])
def test_spokesman_search_matches_oracle(which, request):
    c = request.getfixturevalue(which)
    g = make(c, True)
    n = c.ds.vectors.shape[0]
    _, _, ns = oracle.spokesman(np.bincount(c.ix.cell_of), c.ix.graphs)
    assert g.cross_rows == ns < n
    ix2 = dataclasses.replace(c.ix, cross=oracle.expand_spokesman_cross(c.ix.cell_of, c.ix.graphs, c.ix.cross))
    q, lo, hi = dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi)
    for L, W in ((48, 1), (64, 4), (32, 2)):
        ids, dist = g.search(q, lo, hi, gf.SearchParams(L=L, k=10, width=W))
        ref, ref_d, _ = oracle.search(ix2, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                                      c.offsets, c.cells, c.entry(c.ix.degree), L=L, K=10, width=W)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref)
        assert np.array_equal(dist.cpu().numpy(), ref_d)
    g.close()


def test_spokesman_recall_and_refusals(small):
    c = small
    full, comp = make(c, False), make(c, True)
    q, lo, hi = dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi)
    p = gf.SearchParams(L=64, k=10, width=4)
    r_full = gf.recall(full.search(q, lo, hi, p)[0].cpu().numpy().view(np.uint32), c.gt)
    r_comp = gf.recall(comp.search(q, lo, hi, p)[0].cpu().numpy().view(np.uint32), c.gt)
    print(f"recall@10 full {r_full:.4f} spokesman {r_comp:.4f}, cross rows {comp.cross_rows} of {full.cross_rows}")
    assert r_comp > 0.8 and abs(r_full - r_comp) < 0.1
    assert comp.device_bytes < full.device_bytes
    # the no-allocation entry point searches the compressed index the same way
    f = gf.lib().gf_search_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_float,
                  C.POINTER(gf._SearchParams), C.c_void_p, C.c_void_p, C.c_void_p]
    ref_ids, _ = comp.search(q, lo, hi, p)
    ids = torch.full_like(ref_ids, -7)
    cp = p._c()
    st = f(comp._h, C.c_void_p(q.data_ptr()), C.c_void_p(lo.data_ptr()), C.c_void_p(hi.data_ptr()), q.shape[0], 0.0,
           C.byref(cp), C.c_void_p(ids.data_ptr()), None, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == 0 and torch.equal(ids, ref_ids)
    # batched search over the compressed rows, device-resident and streamed from pinned host
    # memory: the oracle's batched search over the expanded table
    ix2 = dataclasses.replace(c.ix, cross=oracle.expand_spokesman_cross(c.ix.cell_of, c.ix.graphs, c.ix.cross))
    batches = [[0, 1], [2, 3]]
    ref, ref_d, _ = oracle.search(ix2, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                                  c.offsets, c.cells, c.entry(c.ix.degree), L=64, K=10, width=4, batches=batches)
    host = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                           cross_spokesman=True, host_graph=True, keep_fp32=False)
    for g in (comp, host):
        plan = g.plan(q.shape[0])
        plan.build(q, lo, hi)
        ids, dist = plan.search_batched(batches, p)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref)
        assert np.array_equal(dist.cpu().numpy(), ref_d)
        plan.close()
    host.close()
    # a shard keeps its cells' cross blocks in full: compression is refused there
    with pytest.raises(gf.GarfieldError):
        gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                        cross_spokesman=True, shard_cells=[0, 1], keep_fp32=False)
    full.close()
    comp.close()
