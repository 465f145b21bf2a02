"""gf_search_noalloc: the planned search without any allocation, for callers that cannot
allocate device memory while serving queries (see include/garfield.h).  Called through
the C ABI twice in a row; both calls must return exactly what gf_plan_queries +
gf_search return on the same batch (the tests' tolerance for ids and canonical
distances is exact equality), once on an index with few clusters and the graph route,
and once on an index with 128 or more clusters and the exact route (prefilter 0.5),
where gf_search plans with the tensor-core centroid products and gf_search_noalloc with
the CUDA-core top-4 kernel (the tensor-core planner needs a products buffer the fixed
array does not hold): both must produce the same cell orders and results.  Collected
last so that a failing run has already run every other test; it also passes alone in a
fresh process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import garfield_b200 as gf

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _bind():
    lib = gf.lib()
    f = lib.gf_search_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_float,
                  C.POINTER(gf._SearchParams), C.c_void_p, C.c_void_p, C.c_void_p]
    return f


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _two_calls(idx, q, lo, hi, prefilter, params, ref_ids, ref_d):
    f = _bind()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    cp = params._c()
    qnum = q.shape[0]
    for _ in range(2):
        ids = torch.full((qnum, params.k), -7, dtype=torch.int32, device="cuda")
        dist = torch.full((qnum, params.k), -1.0, dtype=torch.float32, device="cuda")
        st = f(idx._h, C.c_void_p(q.data_ptr()), C.c_void_p(lo.data_ptr()), C.c_void_p(hi.data_ptr()), qnum,
               prefilter, C.byref(cp), C.c_void_p(ids.data_ptr()), C.c_void_p(dist.data_ptr()), stream)
        assert st == 0, gf.lib().gf_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids)
        assert torch.equal(dist, ref_d)


@pytest.fixture(scope="module")
def many_clusters():
    """20k x 64 on a 2x2 grid with 160 k-means clusters (the tensor-core planner's range)."""
    from conftest import Case
    return Case(20000, 64, 50, 300, (2, 2), 0.10, R=16, E=2, C=160, seed=31)


def test_noalloc_matches_planned_search_exact_route_many_clusters(many_clusters):
    c = many_clusters
    assert int(c.ix.labels.max()) + 1 >= 128
    idx = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                          l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                          degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels)
    q, lo, hi = _dev(c.ds.queries), _dev(c.ds.lo), _dev(c.ds.hi)
    params = gf.SearchParams(L=64, k=10)
    plan = idx.plan(q.shape[0])
    plan.build(q, lo, hi, 0.5)
    ref_ids, ref_d = plan.search(params)
    torch.cuda.synchronize()
    assert plan.stats()["n_exact"] > 0
    _two_calls(idx, q, lo, hi, 0.5, params, ref_ids, ref_d)
    plan.close()
    idx.close()


def test_noalloc_matches_planned_search(small):
    c = small
    idx = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                          l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                          degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels)
    q, lo, hi = _dev(c.ds.queries), _dev(c.ds.lo), _dev(c.ds.hi)
    qnum = q.shape[0]
    params = gf.SearchParams(L=64, k=10)
    ref_ids, ref_d = idx.search(q, lo, hi, params)
    torch.cuda.synchronize()
    f = _bind()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    cp = params._c()
    for _ in range(2):
        ids = torch.full((qnum, 10), -7, dtype=torch.int32, device="cuda")
        dist = torch.full((qnum, 10), -1.0, dtype=torch.float32, device="cuda")
        st = f(idx._h, C.c_void_p(q.data_ptr()), C.c_void_p(lo.data_ptr()), C.c_void_p(hi.data_ptr()), qnum, 0.0,
               C.byref(cp), C.c_void_p(ids.data_ptr()), C.c_void_p(dist.data_ptr()), stream)
        assert st == 0, gf.lib().gf_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids)
        assert torch.equal(dist, ref_d)
    # a batch larger than the fixed working memory is refused with a clear message
    big = 200_000
    qb = torch.zeros((big, c.ds.vectors.shape[1]), device="cuda")
    bb = torch.zeros((big, 2), device="cuda")
    ib = torch.zeros((big, 10), dtype=torch.int32, device="cuda")
    st = f(idx._h, C.c_void_p(qb.data_ptr()), C.c_void_p(bb.data_ptr()), C.c_void_p(bb.data_ptr()), big, 0.0,
           C.byref(cp), C.c_void_p(ib.data_ptr()), None, stream)
    assert st == 1 and b"split the batch" in gf.lib().gf_last_error()
    idx.close()
