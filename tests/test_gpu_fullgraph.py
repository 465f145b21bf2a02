"""Full-graph post-filter search (gf_index_assemble + gf_search_fullgraph; the reference's
ablation baseline full_graph_search_postfiltering over assemble_edges' graph,
full_graph_search.cuh:179-997) against the oracle restatement: the assembled graph equal,
search ids and canonical distances bit for bit; recall beside the cell-by-cell search."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def fg_entry(n, want):
    """The library's entry positions: std::mt19937 default seed, draw % n, distinct."""
    from conftest import mt19937_stream
    out, seen = [], set()
    for v in mt19937_stream():
        t = v % n
        if t not in seen:
            seen.add(t)
            out.append(t)
            if len(out) == min(want, n):
                break
    return np.array(out, np.uint32)


@pytest.mark.parametrize("which,spokesman", [("small", False), ("odd", False), ("small", True)])
def test_fullgraph_matches_oracle(which, spokesman, request):
    c = request.getfixturevalue(which)
    g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                        cross_spokesman=spokesman)
    g.assemble(2)
    ix = c.ix
    if spokesman:
        import dataclasses
        ix = dataclasses.replace(c.ix, cross=oracle.expand_spokesman_cross(c.ix.cell_of, c.ix.graphs, c.ix.cross))
    n = c.ds.vectors.shape[0]
    entry = fg_entry(n, max(2 * c.ncells, 64))[:c.ix.degree]
    q, lo, hi = dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi)
    plan = g.plan(q.shape[0])
    plan.build(q, lo, hi)
    for L, W in ((64, 1), (48, 4)):
        ids, dist = plan.search_fullgraph(gf.SearchParams(L=L, k=10, width=W))
        ref, ref_d, _ = oracle.search_fullgraph(ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, entry,
                                                L=L, K=10, width=W)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref)
        assert np.array_equal(dist.cpu().numpy(), ref_d)
    gmg, _ = plan.search(gf.SearchParams(L=64, k=10, width=4))
    fullg, _ = plan.search_fullgraph(gf.SearchParams(L=64, k=10, width=4))
    r_g = gf.recall(gmg.cpu().numpy().view(np.uint32), c.gt)
    r_f = gf.recall(fullg.cpu().numpy().view(np.uint32), c.gt)
    print(f"{which}: recall@10 L=64 cell-by-cell {r_g:.4f}, full graph post-filter {r_f:.4f}")
    plan.close()
    g.close()


def test_fullgraph_needs_the_assembled_graph(small):
    c = small
    g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e)
    plan = g.plan(8)
    plan.build(dev(c.ds.queries[:8]), dev(c.ds.lo[:8]), dev(c.ds.hi[:8]))
    with pytest.raises(gf.GarfieldError):
        plan.search_fullgraph(gf.SearchParams(L=32, k=10))
    # an index without clusters plans (cells in id order) and searches; every id is in its box
    ids, _ = plan.search(gf.SearchParams(L=32, k=10))
    ids = ids.cpu().numpy().view(np.uint32)
    for qi in range(8):
        for gid in ids[qi][ids[qi] != gf.NO_ID]:
            a = c.ds.attrs[gid]
            assert np.all(a >= c.ds.lo[qi]) and np.all(a <= c.ds.hi[qi])
    with pytest.raises(gf.GarfieldError):
        g.assemble(0)
    plan.close()
    g.close()
