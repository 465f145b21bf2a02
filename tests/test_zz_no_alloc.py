"""gf_search_noalloc: the planned search without any allocation, for callers that cannot
allocate device memory while serving queries (see include/garfield.h).  Called through
the C ABI twice in a row; both calls must return exactly what gf_plan_queries +
gf_search return on the same batch (the tests' tolerance for ids and canonical
distances is exact equality).  Collected last so that a failing run has already run
every other test; it also passes alone in a fresh process."""
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
