"""CPU oracle self-checks: canonical distances, planning, ordering and the beam-search
restatement's invariants (filter validity, recall against the exact scan)."""
from __future__ import annotations

import itertools

import numpy as np

import oracle


def test_canonical_distances_close_to_float64():
    rng = np.random.default_rng(3)
    for d in (8, 64, 128, 136, 768):
        q = rng.uniform(0, 255, (1, d)).astype(np.float32)
        x = rng.uniform(0, 255, (1, d)).astype(np.float32)
        ref = float(((q.astype(np.float64) - x) ** 2).sum())
        d4 = (d + 3) // 4 * 4
        assert abs(oracle.dist32(oracle.pad(q, 4)[0], oracle.pad(x, 4)[0]) - ref) <= 1e-5 * ref
        d8 = (d + 7) // 8 * 8
        q16, x16 = oracle.f2h(q, d8), oracle.f2h(x, d8)
        qh = q16.view(np.float16).astype(np.float64)
        xh = x16.view(np.float16).astype(np.float64)
        ref16 = float(((qh - xh) ** 2).sum())
        assert abs(oracle.dist16(q16[0], x16[0]) - ref16) <= 1e-5 * ref16
        assert d4 >= d


def test_f2h_rounds_like_ieee_half():
    x = np.array([[0.0, 1.0, 65504.0, 1e-8, 0.333333, 2049.0, 2051.0, -3.5]], np.float32)
    got = oracle.f2h(x, 8).view(np.float16)
    assert np.array_equal(got, x.astype(np.float16))
    got = oracle.f2h(x, 8, alpha=0.01).view(np.float16)
    assert np.array_equal(got, (x * np.float32(0.01)).astype(np.float16))


def _cells_brute(lo, hi, grid, lq, rq):
    """Enumerate every cell and keep those whose slices overlap the box on every dimension."""
    grid = [int(g) for g in grid]
    offs = [int(v) for v in np.concatenate([[0], np.cumsum(grid)])]
    out = []
    for q in range(lo.shape[0]):
        keep = []
        for idx in itertools.product(*[range(g) for g in grid]):
            ok = all(rq[offs[j] + s] >= lo[q, j] and lq[offs[j] + s] <= hi[q, j] for j, s in enumerate(idx))
            if ok:
                pid = 0
                for j, s in enumerate(idx):
                    pid = pid * grid[j] + s
                keep.append(pid)
        out.append(sorted(keep))
    return out


def test_plan_cells_matches_enumeration(small, odd):
    for case in (small, odd):
        ref = _cells_brute(case.ds.lo, case.ds.hi, list(case.ix.grid), case.ix.l_quant, case.ix.r_quant)
        for q in range(case.ds.lo.shape[0]):
            got = case.cells_unordered[case.offsets[q]:case.offsets[q] + case.counts[q]]
            assert list(got) == ref[q]


def test_plan_cells_edge_boxes(small):
    grid, lq, rq = small.ix.grid, small.ix.l_quant, small.ix.r_quant
    # left of the domain, right of it, inverted (l > r inside slice 0: the slice scans of
    # real_dataset_adapter.cuh:168-176 still select slice 0 of dim 0, both slices of dim 1),
    # the whole domain
    lo = np.array([[-10, -10], [20000, 0], [5, 3], [0, 0]], np.int32)
    hi = np.array([[-5, 99999], [30000, 9999], [4, 9999], [9999, 9999]], np.int32)
    counts, offsets, cells = oracle.plan_cells(lo, hi, grid, lq, rq)
    assert [int(c) for c in counts] == [0, 0, 2, small.ncells]


def test_order_cells_by_score(small):
    for q in range(small.ds.queries.shape[0]):
        cl = [int(c) for c in small.cells[small.offsets[q]:small.offsets[q] + small.counts[q]]]
        t4 = small.top4[q]
        scores = [int(sum(small.hist[c, t] for t in t4 if t != oracle.EMPTY)) for c in cl]
        assert all((scores[i], -cl[i]) >= (scores[i + 1], -cl[i + 1]) for i in range(len(cl) - 1))
        # top-4 are the 4 nearest centroids (ties by id) under float64 up to rounding
        d = ((small.centroids.astype(np.float64) - small.ds.queries[q]) ** 2).sum(1)
        assert set(np.argsort(d, kind="stable")[:3]) <= set(t4.tolist())


def test_centroids_and_hist(small):
    lab, cell_of = small.ix.labels, small.ix.cell_of
    for c in range(0, small.centroids.shape[0], 7):
        m = lab == c
        if m.any():
            assert np.allclose(small.centroids[c], small.ds.vectors[m].mean(0), rtol=1e-4, atol=1e-3)
    assert small.hist.sum() == len(lab)
    for cell in range(small.ncells):
        assert small.hist[cell].sum() == (cell_of == cell).sum()


def _valid(ids, attrs, lo, hi):
    for q in range(ids.shape[0]):
        for i in ids[q]:
            if i == oracle.EMPTY:
                continue
            if not ((attrs[i] >= lo[q]) & (attrs[i] <= hi[q])).all():
                return False
    return True


def test_search_filter_and_recall(small):
    c = small
    ent = c.entry(c.ix.degree)
    prev = 0.0
    for L in (16, 64, 160):
        ids, d, st = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                                   c.offsets, c.cells, ent, L=L, K=10)
        assert _valid(ids, c.ds.attrs, c.ds.lo, c.ds.hi)
        r = oracle.recall(ids, c.gt)
        assert r >= prev - 0.02
        prev = r
        assert (np.diff(d, axis=1)[np.isfinite(d[:, 1:])] >= 0).all()
    assert prev >= 0.97


def test_search_width_and_exact_route(small, odd):
    for c in (small, odd):
        ent = c.entry(c.ix.degree)
        ids, _, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                                  c.cells, ent, L=96, K=10, width=3)
        assert _valid(ids, c.ds.attrs, c.ds.lo, c.ds.hi)
        assert oracle.recall(ids, c.gt) >= 0.9
        # postfilter=1: every query scans its cells exactly (fp16 distances)
        ids, _, st = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                                   c.offsets, c.cells, ent, L=16, K=10, postfilter=1)
        assert _valid(ids, c.ds.attrs, c.ds.lo, c.ds.hi)
        assert oracle.recall(ids, c.gt) >= 0.995


def test_prefilter_route_selects_small_boxes(small):
    c = small
    box = oracle.count_in_box(c.ds.attrs, c.ds.lo, c.ds.hi)
    exact_ref = oracle.bruteforce(c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, 10)[0]
    ent = c.entry(c.ix.degree)
    thr = float(np.median(box) / c.ds.vectors.shape[0])
    ids, _, st = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                               c.cells, ent, L=16, K=10, prefilter=thr, box_counts=box)
    small_q = box / c.ds.vectors.shape[0] <= np.float32(thr)
    assert small_q.any()
    assert oracle.recall(ids[small_q], exact_ref[small_q]) >= 0.995


def test_recall_semantics():
    gt = np.array([[1, 2, 3, oracle.EMPTY], [oracle.EMPTY] * 4], np.uint32)
    res = np.array([[3, 9, 1, 7], [5, 6, 7, 8]], np.uint32)
    assert abs(oracle.recall(res, gt) - (2 / 3 + 1.0) / 2) < 1e-12


def test_batched_search_properties(small, odd):
    """orc_search_batched: one batch of every cell is the plain search; any split keeps
    results valid and sorted; the exact route stays exact under any split."""
    for c in (small, odd):
        ent = c.entry(c.ix.degree)
        args = (c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets, c.cells, ent)
        ids0, d0, st0 = oracle.search(*args, L=48, K=10)
        ids1, d1, st1 = oracle.search(*args, L=48, K=10, batches=[list(range(c.ncells))])
        assert (ids0 == ids1).all() and (d0 == d1).all() and (st0 == st1).all()
        rng = np.random.default_rng(7)
        perm = rng.permutation(c.ncells)
        split = [sorted(perm[: c.ncells // 2].tolist()), sorted(perm[c.ncells // 2:].tolist())]
        ids2, d2, _ = oracle.search(*args, L=48, K=10, batches=split)
        assert _valid(ids2, c.ds.attrs, c.ds.lo, c.ds.hi)
        assert (np.diff(d2, axis=1)[np.isfinite(d2[:, 1:])] >= 0).all()
        assert oracle.recall(ids2, c.gt) >= 0.85  # splits lose cross-cell reuse
        # exact route: the merge of per-batch exact lists is the exact list
        ids3, _, _ = oracle.search(*args, L=16, K=10, postfilter=1, batches=[[x] for x in perm.tolist()])
        ids4, _, _ = oracle.search(*args, L=16, K=10, postfilter=1)
        assert (ids3 == ids4).all()
        # a cell searched in no batch contributes nothing
        ids5, _, _ = oracle.search(*args, L=16, K=10, postfilter=1, batches=[[0]])
        in0 = np.isin(ids5, np.flatnonzero(c.ix.cell_of == 0)) | (ids5 == oracle.EMPTY)
        assert in0.all()


def test_nan_centroid_ranks_last():
    """An empty cluster's 0/0 centroid ranks after every real centroid whatever its id
    (pair_less orders NaN distances after numbers, NaNs by id)."""
    rng = np.random.default_rng(5)
    q = rng.standard_normal((6, 8)).astype(np.float32)
    cent = rng.standard_normal((7, 8)).astype(np.float32)
    for gap in (0, 2, 6):
        c2 = cent.copy()
        c2[gap] = np.nan
        hist = np.ones((1, 7), np.uint32)
        counts = np.ones(6, np.uint32)
        offsets = np.arange(6, dtype=np.uint32)
        cells = np.zeros(6, np.uint32)
        _, top4 = oracle.order_cells(q, c2, hist, counts, offsets, cells)
        assert not (top4 == gap).any()
        d = ((q[:, None, :] - c2[None]) ** 2).sum(-1)
        d[:, gap] = np.inf
        assert np.array_equal(top4, np.argsort(d, axis=1, kind="stable")[:, :4].astype(np.uint32))
    c3 = np.full((5, 8), np.nan, np.float32)
    c3[1] = 0.0
    _, top4 = oracle.order_cells(q, c3, np.ones((1, 5), np.uint32), counts, offsets, cells)
    assert (top4 == np.array([1, 0, 2, 3], np.uint32)).all()


def test_assemble_restates_assemble_edges():
    """orc_assemble (full_graph_search.cuh:984-997) on a hand-checked slot layout: own cell's
    first `reserve` graph neighbours in the own slot block, first `reserve` cross edges in the
    others, all as positions."""
    from conftest import Case
    c = Case(3000, 16, 10, 4, (2, 2), 0.2, R=8, E=2, C=10, seed=5)
    fg = oracle.assemble(c.ix, 2)
    order = np.argsort(c.ix.cell_of, kind="stable")
    seg = np.concatenate([[0], np.cumsum(np.bincount(c.ix.cell_of, minlength=4))])
    for pos in (0, 5, 1500, 2999):
        g = order[pos]
        own = int(c.ix.cell_of[g])
        for j in range(4):
            for e in range(2):
                v = fg[pos, j * 2 + e]
                if j == own:
                    loc = c.ix.graphs[pos, e]
                else:
                    loc = c.ix.cross[g, j * 2 + e]
                assert v == seg[j] + loc
