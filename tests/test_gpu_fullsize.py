"""Parity at the benchmark's full size (config 2: 1M x 128, 4x4 grid, R=32, E=2, C=1000,
10k queries at 10% selectivity): the planner's 4 nearest centroids and cell order, and the
search's ids and distances for every query, against the oracle on the same index.  The
index is built on the GPU (about 40 s); the oracle's planner and search take seconds."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def config2():
    from garfield_b200 import indexbuild, synth
    ds = synth.config2(seed=20261201)
    ix = indexbuild.build(ds.vectors, ds.attrs, ds.grid, R=32, E=2, C=1000, seed=20261201, device="cuda:0")
    torch.cuda.synchronize()
    return ds, ix


def test_config2_planner_and_search_match_oracle(config2):
    from conftest import mt_entry
    ds, ix = config2
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid,
                            l_quant=ix.l_quant, r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs,
                            degree=ix.degree, cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels,
                            keep_fp32=False)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    plan = index.plan(ds.queries.shape[0])
    plan.build(dev(ds.queries), dev(ds.lo), dev(ds.hi))
    counts, offsets, cells, top4, _ = plan.read()
    ncells = int(np.prod(ix.grid))
    # the cell intersection on its own: the oracle's cell lists from the boxes and quantiles
    ocounts, ooffsets, ounordered = oracle.plan_cells(ds.lo, ds.hi, ix.grid, ix.l_quant, ix.r_quant)
    assert np.array_equal(counts, ocounts) and np.array_equal(offsets, ooffsets)
    cent, hist = oracle.cluster_info(ds.vectors, ix.labels, ix.cell_of, ncells)
    ocells, otop4 = oracle.order_cells(ds.queries, cent, hist, ocounts, ooffsets, ounordered.copy())
    assert np.array_equal(top4, otop4) and np.array_equal(cells, ocells)
    ids, dist = plan.search(gf.SearchParams(L=40, k=10, width=4))
    st = plan.stats()
    assert st["n_timeouts"] == 0
    ent = mt_entry(ix.degree, int(np.bincount(ix.cell_of, minlength=ncells).min()))
    ref_ids, ref_d, _ = oracle.search(ix, ds.vectors, ds.attrs, ds.queries, ds.lo, ds.hi, counts, offsets, cells,
                                      ent, L=40, K=10, width=4)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_ids)
    assert np.array_equal(dist.cpu().numpy(), ref_d)
