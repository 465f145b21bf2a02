"""GPU parity: every CUDA stage through the C ABI against the CPU oracle on the same
inputs.  Integer outputs (ids, cell lists, counters) must match exactly; distances are
computed in the same fixed fp32 order on both sides and must match bit for bit."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def make_index(c, alpha=1.0):
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                           f2h_factor=alpha, keep_fp32=True)


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


@pytest.fixture(scope="module")
def g_small(small):
    return make_index(small)


@pytest.fixture(scope="module")
def g_odd(odd):
    return make_index(odd)


def as_u32(t):
    return t.cpu().numpy().view(np.uint32) if t.dtype == torch.int32 else t.cpu().numpy().astype(np.uint32)


def test_index_info_and_entry_points(small, g_small):
    from conftest import mt_entry
    assert g_small.n == small.ds.vectors.shape[0] and g_small.n_cells == small.ncells
    minc = int(np.bincount(small.ix.cell_of).min())
    assert g_small.min_cell_size == minc
    assert np.array_equal(g_small.entry_points(32), mt_entry(32, minc))


@pytest.mark.parametrize("which", ["small", "odd"])
def test_bruteforce_bit_exact(which, request):
    c = request.getfixturevalue(which)
    g = request.getfixturevalue("g_" + which)
    for k in (10, 37):
        ids, dist = g.bruteforce(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), k)
        ref_ids, ref_d = oracle.bruteforce(c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, k)
        assert np.array_equal(as_u32(ids), ref_ids)
        assert np.array_equal(dist.cpu().numpy(), ref_d)


@pytest.mark.parametrize("which", ["small", "odd"])
def test_plan_matches_oracle(which, request):
    c = request.getfixturevalue(which)
    g = request.getfixturevalue("g_" + which)
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), prefilter=0.5)
    counts, offsets, cells, top4, box = plan.read()
    assert np.array_equal(counts, c.counts) and np.array_equal(offsets, c.offsets)
    assert np.array_equal(top4, c.top4)
    assert np.array_equal(cells, c.cells)
    assert np.array_equal(box, oracle.count_in_box(c.ds.attrs, c.ds.lo, c.ds.hi))


def _oracle_search(c, **kw):
    ent = c.entry(kw.pop("n_entry", c.ix.degree))
    return oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                         c.cells, ent, **kw)


@pytest.mark.parametrize("which", ["small", "odd"])
@pytest.mark.parametrize("L,width", [(16, 1), (64, 1), (160, 1), (64, 2), (96, 4)])
def test_search_matches_oracle(which, L, width, request):
    c = request.getfixturevalue(which)
    g = request.getfixturevalue("g_" + which)
    params = gf.SearchParams(L=L, k=10, width=width)
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search(params)
    st = plan.stats()
    ref_ids, ref_d, ref_st = _oracle_search(c, L=L, K=10, width=width)
    got = as_u32(ids)
    assert np.array_equal(got, ref_ids), np.argwhere(got != ref_ids)[:5]
    assert np.array_equal(dist.cpu().numpy(), ref_d)
    assert st["n_exp"] == ref_st[1] and st["n_cross"] == ref_st[2] and st["n_hops"] == ref_st[3]
    assert st["n_queries"] == c.ds.queries.shape[0]


def test_exact_and_prefilter_routes(small, g_small):
    c = small
    q = c.ds.queries.shape[0]
    plan = g_small.plan(q)
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search(gf.SearchParams(L=16, k=10, postfilter=1))
    ref_ids, ref_d, _ = _oracle_search(c, L=16, K=10, postfilter=1)
    assert np.array_equal(as_u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    assert plan.stats()["n_exact"] == int((c.counts >= 1).sum())
    box = oracle.count_in_box(c.ds.attrs, c.ds.lo, c.ds.hi)
    thr = float(np.median(box) / c.ds.vectors.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), prefilter=thr)
    ids, dist = plan.search(gf.SearchParams(L=32, k=10))
    ref_ids, ref_d, _ = _oracle_search(c, L=32, K=10, prefilter=thr, box_counts=box)
    assert np.array_equal(as_u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)


def test_search_host_matches_device(small, g_small):
    c = small
    q = c.ds.queries.shape[0]
    plan = g_small.plan(q)
    params = gf.SearchParams(L=48, k=10)
    ids_h, d_h = g_small.search_host(c.ds.queries.astype(np.float32), c.ds.lo.astype(np.float32),
                                     c.ds.hi.astype(np.float32), plan, params, with_dist=True)
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search(params)
    assert np.array_equal(ids_h, as_u32(ids)) and np.array_equal(d_h, dist.cpu().numpy())


def test_filter_validity_and_recall(small, g_small):
    c = small
    ids, _ = g_small.search(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), gf.SearchParams(L=160, k=10))
    ids = as_u32(ids)
    for q in range(ids.shape[0]):
        for i in ids[q]:
            if i != gf.NO_ID:
                assert ((c.ds.attrs[i] >= c.ds.lo[q]) & (c.ds.attrs[i] <= c.ds.hi[q])).all()
    assert oracle.recall(ids, c.gt) >= 0.97


def test_edge_cases(small, g_small):
    c = small
    q = np.ascontiguousarray(c.ds.queries[:6])
    lo = np.array([[-9, -9], [20000, 0], [0, 0], [c.ds.attrs[7, 0], c.ds.attrs[7, 1]], [5, 3], [0, 0]], np.int32)
    hi = np.array([[-5, 99], [30000, 99], [9999, 9999], [c.ds.attrs[7, 0], c.ds.attrs[7, 1]], [4, 9999],
                   [9999, 9999]], np.int32)
    params = gf.SearchParams(L=20, k=20)
    ids, dist = g_small.search(dev(q), dev(lo), dev(hi), params)
    ids = as_u32(ids)
    assert (ids[0] == gf.NO_ID).all() and (ids[1] == gf.NO_ID).all() and (ids[4] == gf.NO_ID).all()
    assert np.isinf(dist.cpu().numpy()[0]).all()
    # a box around one point's attributes: only points with exactly those attributes qualify
    same = np.where((c.ds.attrs == c.ds.attrs[7]).all(1))[0]
    got = [int(v) for v in ids[3] if v != gf.NO_ID]
    assert set(got) <= set(same.tolist())
    # L == k and a single query
    ids1, _ = g_small.search(dev(q[:1]), dev(lo[2:3]), dev(hi[2:3]), gf.SearchParams(L=10, k=10))
    assert ids1.shape == (1, 10)
    with pytest.raises(gf.GarfieldError):
        g_small.search(dev(q[:1]), dev(lo[2:3]), dev(hi[2:3]), gf.SearchParams(L=5, k=10))


def test_f2h_factor(small):
    c = small
    g = make_index(c, alpha=0.01)
    params = gf.SearchParams(L=64, k=10)
    ids, dist = g.search(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), params)
    ref_ids, ref_d, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                                      c.offsets, c.cells, c.entry(c.ix.degree), L=64, K=10, alpha=0.01)
    assert np.array_equal(as_u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    g.close()


def test_plan_may_outlive_its_index(small):
    """Destroying a plan after its index (as a garbage collector may order them) leaves no
    error behind: the next index builds."""
    g = make_index(small)
    plan = g.plan(8)
    g.close()
    plan.close()
    make_index(small).close()


def test_staging_wait_timeout_is_reported(small, g_small):
    """The bounded row-staging wait: with the test hook no staging batch can complete, the
    waits give up, the warps stop, the counter and gf_search_host report it, and the
    context stays usable for the next search."""
    c = small
    plan = g_small.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    plan.search(gf.SearchParams(L=32, k=10, test_wait=64))
    assert plan.stats()["n_timeouts"] > 0
    with pytest.raises(gf.GarfieldError) as e:
        g_small.search_host(c.ds.queries, c.ds.lo.astype(np.float32), c.ds.hi.astype(np.float32), plan,
                            gf.SearchParams(L=32, k=10, test_wait=64))
    assert e.value.status == 6
    ids, dist = plan.search(gf.SearchParams(L=32, k=10))
    assert plan.stats()["n_timeouts"] == 0
    ref_ids, ref_d, _ = _oracle_search(c, L=32, K=10)
    assert np.array_equal(as_u32(ids), ref_ids)


def test_graph_rows_not_a_multiple_of_16_bytes():
    """Degree 18 (72-byte rows): the picks' neighbour rows are read with plain loads instead
    of bulk copies; results and counters still equal the oracle's."""
    from conftest import Case
    c = Case(8000, 48, 30, 200, (2, 2), 0.2, R=18, E=2, C=30, seed=41)
    assert c.ix.degree % 4 != 0
    g = make_index(c)
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    for L, width in ((32, 1), (64, 4)):
        ids, dist = plan.search(gf.SearchParams(L=L, k=10, width=width))
        st = plan.stats()
        ref_ids, ref_d, ref_st = _oracle_search(c, L=L, K=10, width=width)
        assert np.array_equal(as_u32(ids), ref_ids)
        assert np.array_equal(dist.cpu().numpy(), ref_d)
        assert st["n_exp"] == ref_st[1] and st["n_cross"] == ref_st[2] and st["n_hops"] == ref_st[3]


@pytest.mark.parametrize("which", ["small", "odd"])
def test_box_counts_from_attribute_tiles(which, request):
    """The plan's box counts (prefilter) come from the attribute tiles: tiles inside a box
    add their counts, tiles that meet it are tested row by row.  Against the oracle's scan
    of every point, on the queries' boxes and on edge boxes: the whole domain, empty boxes,
    boxes that are one point, boxes whose bounds are attribute values of the data."""
    c = request.getfixturevalue(which)
    g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                        keep_fp32=False)
    rng = np.random.default_rng(3)
    a = c.ds.attrs.shape[1]
    at = c.ds.attrs
    pts = at[rng.integers(0, at.shape[0], 40)]
    lo = np.concatenate([c.ds.lo, np.full((1, a), -1), np.full((1, a), 5), pts, np.minimum(pts, at[:40]),
                         at[rng.integers(0, at.shape[0], 40)] - 1]).astype(np.int32)
    hi = np.concatenate([c.ds.hi, np.full((1, a), 20000), np.full((1, a), 4), pts, np.maximum(pts, at[:40]),
                         at[rng.integers(0, at.shape[0], 40)] + 300]).astype(np.int32)
    q = np.repeat(c.ds.queries[:1], lo.shape[0], 0)
    plan = g.plan(lo.shape[0])
    plan.build(dev(q), dev(lo), dev(hi), prefilter=0.5)
    box = plan.read()[4]
    assert np.array_equal(box, oracle.count_in_box(c.ds.attrs, lo, hi))
    assert box[c.ds.lo.shape[0]] == at.shape[0] and box[c.ds.lo.shape[0] + 1] == 0
    plan.close()
    g.close()


def test_exact_route_rows_outside_their_cells(small):
    """The exact route scans the in-box rows of the query's cells.  When a row's attributes
    fall outside its cell's slice ranges (fractional attributes between integer quantiles,
    or a cell_of that disagrees with the ranges), that set differs from "every in-box row of
    the index", so the search must keep the cell scan: boxes inside the gap between two
    slices meet no cell and return nothing, like the oracle's."""
    c = small
    attrs = c.ds.attrs.astype(np.float32).copy()
    g0 = int(c.ix.grid[0])
    lq, rq = c.ix.l_quant[:g0].astype(np.float32), c.ix.r_quant[:g0].astype(np.float32)
    slice0 = c.ix.slices[:, 0]
    edge = attrs[:, 0] == rq[slice0]               # rows on the upper edge of their slice
    edge &= slice0 < g0 - 1
    attrs[edge, 0] += 0.5                          # now strictly between two slices
    assert edge.sum() > 0
    idx = gf.Index.create(vectors=c.ds.vectors, attrs=attrs, grid=c.ix.grid, l_quant=c.ix.l_quant,
                          r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs, degree=c.ix.degree,
                          cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels, keep_fp32=True)
    q = c.ds.queries.shape[0]
    lo = c.ds.lo.astype(np.float32).copy()
    hi = c.ds.hi.astype(np.float32).copy()
    # half of the boxes sit in the gap above slice 0 on dimension 0
    gap = np.arange(q) % 2 == 0
    lo[gap, 0], hi[gap, 0] = rq[0] + 0.25, rq[0] + 0.75
    lo[gap, 1], hi[gap, 1] = -1e9, 1e9
    counts, offsets, cells_u = oracle.plan_cells(lo, hi, c.ix.grid, c.ix.l_quant, c.ix.r_quant)
    assert (counts[gap] == 0).all()
    cells, _ = oracle.order_cells(c.ds.queries, c.centroids, c.hist, counts, offsets, cells_u)
    box = oracle.count_in_box(attrs, lo, hi)
    assert (box[gap] > 0).sum() > 0                 # rows of the index do lie in those boxes
    plan = idx.plan(q)
    plan.build(dev(c.ds.queries), dev(lo), dev(hi), prefilter=1.0)
    ids, dist = plan.search(gf.SearchParams(L=32, k=10))
    ent = c.entry(c.ix.degree)
    ref_ids, ref_d, _ = oracle.search(c.ix, c.ds.vectors, attrs, c.ds.queries, lo, hi, counts, offsets, cells, ent,
                                      L=32, K=10, prefilter=1.0, box_counts=box)
    assert np.array_equal(as_u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    assert (as_u32(ids)[gap] == gf.NO_ID).all()
    plan.close()
    idx.close()
