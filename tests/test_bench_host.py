"""Host logic of bench.py that needs no GPU: the cell-major renumbering used to run the
reference's binary and ours on the same files (the reference's load_clustering histograms
cells as id / 62500, tools.cuh:590, so ids must be cell-major), and the per-rank query
streams of the multi-GPU mode."""
from __future__ import annotations

import numpy as np

import bench
import oracle


def test_cell_major_renumbering_keeps_the_index():
    from garfield_b200 import indexbuild, synth
    ds = synth.make(6000, 16, 12, 40, (2, 2), 0.3, seed=9, stratified=False)
    ix = indexbuild.build(ds.vectors, ds.attrs, ds.grid, R=8, E=2, C=12, seed=9, device="cpu")
    gt, _ = oracle.bruteforce(ds.vectors, ds.attrs, ds.queries, ds.lo, ds.hi, 10)
    ds2, ix2, gt2 = bench._cell_major(ds, ix, gt)
    order = np.argsort(ix.cell_of, kind="stable")
    assert np.all(np.diff(ix2.cell_of.astype(np.int64)) >= 0)           # ids are cell-major
    assert np.array_equal(ds2.vectors, ds.vectors[order]) and np.array_equal(ds2.attrs, ds.attrs[order])
    assert np.array_equal(ix2.graphs, ix.graphs)                         # positions and local ids unchanged
    assert np.array_equal(ix2.cross, ix.cross[order])
    inv = np.empty_like(order)
    inv[order] = np.arange(order.size)
    assert np.array_equal(gt2, np.where(gt == 0xFFFFFFFF, gt, inv[np.minimum(gt, order.size - 1)]))
    # the exact answer of the renumbered data is the renumbered answer (ties aside)
    gt_b, _ = oracle.bruteforce(ds2.vectors, ds2.attrs, ds2.queries, ds2.lo, ds2.hi, 10)
    assert (gt_b == gt2).mean() > 0.99
    # the graph search over the renumbered index visits the same positions: same answer
    def search(d, x):
        counts, offsets, cells = oracle.plan_cells(d.lo, d.hi, x.grid, x.l_quant, x.r_quant)
        cent, hist = oracle.cluster_info(d.vectors, x.labels, x.cell_of, 4)
        cells, _ = oracle.order_cells(d.queries, cent, hist, counts, offsets, cells)
        from conftest import mt_entry
        ent = mt_entry(8, int(np.bincount(x.cell_of, minlength=4).min()))
        return oracle.search(x, d.vectors, d.attrs, d.queries, d.lo, d.hi, counts, offsets, cells, ent, L=32, K=10)
    ids, dist, _ = search(ds, ix)
    ids2, dist2, _ = search(ds2, ix2)
    assert np.array_equal(np.where(ids == 0xFFFFFFFF, ids, inv[np.minimum(ids, order.size - 1)]), ids2)
    assert np.array_equal(dist, dist2)
