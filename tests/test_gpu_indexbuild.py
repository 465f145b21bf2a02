"""Index construction on the GPU: the cross-cell edges that large indexes get from this
library's own beam search of each cell's graph (indexbuild.cross_edges_by_search, the
reference's cagra.search-based global graph, indexbuild/global_graph_build.py:116-157)
against the exact E nearest points per cell."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_cross_edges_by_search_match_exact(small):
    from garfield_b200 import indexbuild
    c = small
    ix = c.ix
    P = int(np.prod(ix.grid))
    E = ix.cross_e
    got = indexbuild.cross_edges_by_search(c.ds.vectors, c.ds.attrs, ix.grid, ix.l_quant, ix.r_quant, ix.cell_of,
                                           ix.graphs, ix.degree, E, L=32, width=4, chunk=4096, device="cuda")
    assert got.shape == ix.cross.shape and got.dtype == np.uint32
    sizes = np.bincount(ix.cell_of, minlength=P)
    seg = np.concatenate([[0], np.cumsum(sizes)])
    order = np.argsort(ix.cell_of, kind="stable")
    local = np.empty(len(order), np.int64)
    local[order] = np.arange(len(order)) - seg[ix.cell_of[order]]
    n = c.ds.vectors.shape[0]
    own = ix.cell_of.astype(np.int64)
    hits = total = 0
    for cell in range(P):
        cols = slice(cell * E, (cell + 1) * E)
        other = own != cell
        assert (got[other, cols] < sizes[cell]).all()          # local ids of that cell
        g, x = got[other, cols], ix.cross[other, cols]          # ix.cross: exact E nearest
        hits += sum(len(set(a) & set(b)) for a, b in zip(g.tolist(), x.tolist()))
        total += x.size
        # the first found point is at least as far as the exact nearest
        pts = c.ds.vectors[order[seg[cell] + g[:, 0]]]
        ref = c.ds.vectors[order[seg[cell] + x[:, 0]]]
        q = c.ds.vectors[other]
        assert (((q - pts) ** 2).sum(1) >= ((q - ref) ** 2).sum(1) * (1 - 1e-4) - 1e-3).all()
    assert hits / total >= 0.9
    for j in range(E):  # own-cell slots hold the point's own local id
        assert np.array_equal(got[np.arange(n), own * E + j], local.astype(np.uint32))
