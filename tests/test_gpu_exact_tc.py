"""gf_search_params.exact_tc: queries that take the exact route (postfilter, plan prefilter)
are answered by the tensor-core exact scan instead of the fp16 warp scan.  Their rows must
equal the oracle's exact filtered scan over the fp32 rows (ids and canonical distances bit
for bit); every other row must equal the oracle's graph search; n_exact counts the routed
queries; the entry points that cannot take the route refuse it."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def make(c, **kw):
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                           f2h_factor=1.0, **kw)


def exact_rows(c, prefilter, postfilter):
    """The search kernel's routing rule on the oracle's plan."""
    box = oracle.count_in_box(c.ds.attrs, c.ds.lo, c.ds.hi)
    n = c.ds.vectors.shape[0]
    share = (box.astype(np.float64) / n).astype(np.float32)
    ex = (c.counts > 0) & ((c.counts >= postfilter) | ((prefilter > 0) & (share <= np.float32(prefilter))))
    return ex, box


@pytest.mark.parametrize("which,k", [("small", 10), ("odd", 10), ("small", 40)])
def test_exact_tc_rows_match_oracle(which, k, request):
    c = request.getfixturevalue(which)
    g = make(c, keep_fp32=True)
    q = c.ds.queries.shape[0]
    box = oracle.count_in_box(c.ds.attrs, c.ds.lo, c.ds.hi)
    thr = float(np.median(box) / c.ds.vectors.shape[0])
    ex, _ = exact_rows(c, thr, 0xFFFFFFFF)
    assert 0 < ex.sum() < q
    plan = g.plan(q)
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), prefilter=thr)
    L = max(48, k)
    ids, dist = plan.search(gf.SearchParams(L=L, k=k, exact_tc=1))
    st = plan.stats()
    ids = ids.cpu().numpy().view(np.uint32)
    dist = dist.cpu().numpy()
    bf_ids, bf_d = oracle.bruteforce(c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, k)
    ref_ids, ref_d, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                                      c.offsets, c.cells, c.entry(c.ix.degree), L=L, K=k, prefilter=thr,
                                      box_counts=box)
    assert np.array_equal(ids[ex], bf_ids[ex]) and np.array_equal(dist[ex], bf_d[ex])
    assert np.array_equal(ids[~ex], ref_ids[~ex]) and np.array_equal(dist[~ex], ref_d[~ex])
    assert st["n_exact"] == int(ex.sum()) and st["n_queries"] == q
    # gf_search_host takes the same route
    h_ids, h_d = g.search_host(c.ds.queries.astype(np.float32), c.ds.lo.astype(np.float32),
                               c.ds.hi.astype(np.float32), plan, gf.SearchParams(L=L, k=k, exact_tc=1),
                               prefilter=thr, with_dist=True)
    assert np.array_equal(h_ids, ids) and np.array_equal(h_d, dist)
    plan.close()
    g.close()


def test_exact_tc_postfilter_routes_every_query(small):
    c = small
    g = make(c, keep_fp32=True)
    q = c.ds.queries.shape[0]
    plan = g.plan(q)
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search(gf.SearchParams(L=16, k=10, postfilter=1, exact_tc=1))
    ex, _ = exact_rows(c, 0.0, 1)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32)[ex], c.gt[ex])
    assert np.array_equal(dist.cpu().numpy()[ex], c.gt_d[ex])
    assert plan.stats()["n_exact"] == int(ex.sum())
    plan.close()
    g.close()


def test_exact_tc_refusals(small):
    c = small
    q = c.ds.queries.shape[0]
    p = gf.SearchParams(L=32, k=10, postfilter=1, exact_tc=1)
    g16 = make(c, keep_fp32=False)  # no fp32 rows: no tensor-core copy
    plan = g16.plan(q)
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    with pytest.raises(gf.GarfieldError):
        plan.search(p)
    plan.close()
    g16.close()
    g = make(c, keep_fp32=True)
    plan = g.plan(q)
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    with pytest.raises(gf.GarfieldError):
        plan.search(gf.SearchParams(L=200, k=129, postfilter=1, exact_tc=1))
    with pytest.raises(gf.GarfieldError):
        plan.search_batched([[0, 1], [2, 3]], p)
    f = gf.lib().gf_search_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_float,
                  C.POINTER(gf._SearchParams), C.c_void_p, C.c_void_p, C.c_void_p]
    qd, lo, hi = dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi)
    ids = torch.empty((q, 10), dtype=torch.int32, device="cuda")
    cp = p._c()
    st = f(g._h, C.c_void_p(qd.data_ptr()), C.c_void_p(lo.data_ptr()), C.c_void_p(hi.data_ptr()), q, 0.0,
           C.byref(cp), C.c_void_p(ids.data_ptr()), None, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st != 0
    # a normal search on the same plan is unaffected by the refused calls
    ids, _ = plan.search(gf.SearchParams(L=32, k=10))
    ref, _, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                              c.cells, c.entry(c.ix.degree), L=32, K=10)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref)
    plan.close()
    g.close()


def test_route_by_cost(small):
    """gf_search_params.route = 1: a query also goes to the tensor-core exact scan when its
    box count is below GF_ROUTE_ROWS_PER_SLOT (150) x cells x (L + 64).  The rule on the
    host must mark the same queries (n_exact), and their rows must be the exact scan's."""
    c = small
    g = make(c, keep_fp32=True)
    q = c.ds.queries.shape[0]
    L, k = 48, 10
    lo, hi = c.ds.lo.copy(), c.ds.hi.copy()
    lo[::3] = -1, -1          # a third of the boxes cover the whole domain
    hi[::3] = 20000, 20000
    counts, _, _ = oracle.plan_cells(lo, hi, c.ix.grid, c.ix.l_quant, c.ix.r_quant)
    box = oracle.count_in_box(c.ds.attrs, lo, hi)
    ex = (counts > 0) & (box.astype(np.int64) < 150 * counts.astype(np.int64) * (L + 64))
    plan = g.plan(q)
    plan.build(dev(c.ds.queries), dev(lo), dev(hi), prefilter=1e-9)
    ids, dist = plan.search(gf.SearchParams(L=L, k=k, exact_tc=1, route=1))
    assert plan.stats()["n_exact"] == int(ex.sum()) > 0
    bf_ids, bf_d = oracle.bruteforce(c.ds.vectors, c.ds.attrs, c.ds.queries, lo, hi, k)
    ids, dist = ids.cpu().numpy().view(np.uint32), dist.cpu().numpy()
    assert np.array_equal(ids[ex], bf_ids[ex]) and np.array_equal(dist[ex], bf_d[ex])
    # without the tensor-core scan the option is refused
    with pytest.raises(gf.GarfieldError):
        plan.search(gf.SearchParams(L=L, k=k, route=1))
    # a plan without box counts: the search estimates them from the attribute tiles; every
    # row is the exact scan's or the graph search's
    plan.build(dev(c.ds.queries), dev(lo), dev(hi))
    ids2, dist2 = plan.search(gf.SearchParams(L=L, k=k, exact_tc=1, route=1))
    n2 = plan.stats()["n_exact"]
    ids2, dist2 = ids2.cpu().numpy().view(np.uint32), dist2.cpu().numpy()
    g_ids, g_d = plan.search(gf.SearchParams(L=L, k=k))
    g_ids, g_d = g_ids.cpu().numpy().view(np.uint32), g_d.cpu().numpy()
    exact_rows = np.all(ids2 == bf_ids, 1) & np.all(dist2 == bf_d, 1)
    graph_rows = np.all(ids2 == g_ids, 1) & np.all(dist2 == g_d, 1)
    assert (exact_rows | graph_rows).all() and n2 >= int(ex.sum()) * 0.5
    plan.close()
    g.close()
