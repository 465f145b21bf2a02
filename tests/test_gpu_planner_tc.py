"""The tensor-core planner (gf_centroid_tc.cu, used when an index has >= 256 centroids):
tf32 products on tcgen05, an error bound, and an exact re-rank must give exactly the
oracle's 4 nearest centroids and cell order (orc_order_cells, canonical fp32 distances)."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.float32)


@pytest.fixture(scope="module")
def many_clusters():
    from conftest import Case
    return [Case(12000, 64, 60, 500, (2, 2), 0.15, R=16, E=2, C=300, seed=31),
            Case(9000, 100, 50, 400, (2, 2, 2), 0.2, R=16, E=2, C=260, seed=32, stratified=False)]


def test_tensor_core_top4_matches_oracle(many_clusters):
    for c in many_clusters:
        g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                            l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                            degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                            keep_fp32=False)
        assert g.n_clusters and int(c.ix.labels.max()) + 1 >= 256
        plan = g.plan(c.ds.queries.shape[0])
        plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
        counts, offsets, cells, top4, _ = plan.read()
        assert np.array_equal(top4, c.top4)
        assert np.array_equal(cells, c.cells)
        ids, _ = plan.search(gf.SearchParams(L=48, k=10))
        st = plan.stats()
        assert st["n_plan_fallbacks"] == 0 and st["n_timeouts"] == 0
        # the error bound must stay tight: a wrong product tile would let many centroids through
        assert st["n_plan_reranked"] <= 16 * c.ds.queries.shape[0]
        ent = c.entry(c.ix.degree)
        ref, _, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                                  c.cells, ent, L=48, K=10)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref)


def test_tensor_core_planner_on_shards(many_clusters):
    """Shard indexes plan only the queries with two or more of their cells (gathered rows,
    a device-side count): the same top4 and order for those, and merged shard searches
    equal the oracle's batched search with the shards as batches.  Every second query's
    box is shrunk to 1 % so that it holds one or two cells; two shards of two cells plan
    some queries each, four shards of one cell plan none."""
    import types
    from conftest import check_shard_plan
    from garfield_b200.dist import shard_cells
    c = many_clusters[0]
    lo, hi = c.ds.lo.copy(), c.ds.hi.copy()
    hi[1::2] = lo[1::2] + (hi[1::2] - lo[1::2]) // 100  # integer bounds, as generated
    counts, offsets, unordered = oracle.plan_cells(lo, hi, c.ix.grid, c.ix.l_quant, c.ix.r_quant)
    cells, top4 = oracle.order_cells(c.ds.queries, c.centroids, c.hist, counts, offsets, unordered.copy())
    want = types.SimpleNamespace(counts=counts, offsets=offsets, cells=cells, top4=top4)
    qnum = c.ds.queries.shape[0]
    for world, lo_planned, hi_planned in ((2, 1, qnum - 1), (4, 0, 0)):
        shards = shard_cells(c.ix.grid, world)
        keys = []
        for sh in shards:
            g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                                l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                                degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                                keep_fp32=False, shard_cells=sh)
            plan = g.plan(qnum)
            plan.build(dev(c.ds.queries), dev(lo), dev(hi))
            _, _, got_cells, got_top4, _ = plan.read()
            n = check_shard_plan(want, sh, got_top4, got_cells)
            assert lo_planned <= n <= hi_planned, (world, sh, n)
            keys.append(plan.search_keys(gf.SearchParams(L=48, k=10)).clone())
            assert plan.stats()["n_plan_fallbacks"] == 0
        ids, _ = g.merge_keys(torch.stack(keys, 0), 10)
        ref, _, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, lo, hi, counts, offsets, cells,
                                  c.entry(c.ix.degree), L=48, K=10, batches=shards)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref)


def _with_empty_cluster(c, gap):
    """c's clustering with label `gap` left empty: its centroid is 0/0 (NaN), as the
    reference's load_clustering computes it, and it must rank after every real centroid."""
    lab = c.ix.labels.astype(np.int32)
    lab = lab + (lab >= gap).astype(np.int32)
    cent, hist = oracle.cluster_info(c.ds.vectors, lab, c.ix.cell_of, c.ncells)
    assert np.isnan(cent[gap]).all()
    cells, top4 = oracle.order_cells(c.ds.queries, cent, hist, c.counts, c.offsets, c.cells_unordered)
    g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=lab, keep_fp32=False)
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    _, _, got_cells, got_top4, _ = plan.read()
    assert not (got_top4 == gap).any()
    assert np.array_equal(got_top4, top4)
    assert np.array_equal(got_cells, cells)
    return plan.stats()


def test_empty_cluster_tensor_core_path(many_clusters):
    st = _with_empty_cluster(many_clusters[0], 5)
    assert st["n_plan_fallbacks"] == 0  # the NaN column neither shrinks U nor floods the candidates


def test_empty_cluster_cuda_core_path(small):
    _with_empty_cluster(small, 3)


def test_non_finite_query_scans_every_centroid(many_clusters):
    """A NaN query has NaN distances to every centroid: the bound rules nothing out, the
    planner re-ranks every centroid and, like the oracle, keeps ids 0..3 (NaNs by id)."""
    c = many_clusters[0]
    qs = c.ds.queries.copy()
    qs[7] = np.nan
    cells, top4 = oracle.order_cells(qs, c.centroids, c.hist, c.counts, c.offsets, c.cells_unordered)
    assert (top4[7] == np.arange(4)).all()
    g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                        keep_fp32=False)
    plan = g.plan(qs.shape[0])
    plan.build(dev(qs), dev(c.ds.lo), dev(c.ds.hi))
    _, _, got_cells, got_top4, _ = plan.read()
    assert np.array_equal(got_top4, top4) and np.array_equal(got_cells, cells)
    assert plan.stats()["n_plan_fallbacks"] == 1
