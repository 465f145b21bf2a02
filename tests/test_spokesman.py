"""Spokesman compression of the cross-cell edges (compress_global_graph_extreme and
save_global_graph_extreme, tools.cuh:917-1038) against the reference's own code: the
fixture golden_spokesman.npz is the file the reference writes for seeded per-cell graphs
(tests/golden/make_golden.py, oracle/ref_spokesman.cu).  CPU only."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

GOLD = Path(__file__).resolve().parent / "golden" / "golden_spokesman.npz"


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_spokesman_ranks_match_the_reference(gold):
    sizes, graphs = gold["sizes"], gold["graphs"]
    _, rank, ns = gf.spokesman(sizes, graphs)
    assert np.array_equal(rank, gold["center_pos"])
    assert ns == int(gold["center_num"].sum())
    ospk, orank, ons = oracle.spokesman(sizes, graphs)
    assert np.array_equal(orank, gold["center_pos"]) and ons == ns
    # a spokesman is its own spokesman and precedes its followers in the same cell
    pos = np.arange(len(ospk))
    assert np.all(ospk <= pos) and np.all(ospk[ospk] == ospk)


def test_compressed_file_is_the_reference_file(gold, tmp_path):
    sizes, graphs, cross_t, E = gold["sizes"], gold["graphs"], gold["cross_t"], int(gold["e"])
    P, n = len(sizes), int(sizes.sum())
    cell_of = np.repeat(np.arange(P, dtype=np.uint32), sizes)  # global order = position order here
    cross = np.ascontiguousarray(cross_t.transpose(1, 0, 2)).reshape(n, P * E)
    cn, co, cp, edges = gf.compress_cross(cell_of, graphs, cross, E)
    assert np.array_equal(cn, gold["center_num"]) and np.array_equal(co, gold["col_offset"])
    assert np.array_equal(cp, gold["center_pos"]) and np.array_equal(edges, gold["edges"])
    path = tmp_path / "global_graph.extreme"
    gf.write_spokesman_graph(path, cn, co, cp, edges)
    assert path.read_bytes() == gold["raw"].tobytes()
    back = gf.read_spokesman_graph(path)
    for a, b in zip(back, (cn, co, cp, edges)):
        assert np.array_equal(a, b)


def test_expanded_cross_edges_follow_the_spokesman(gold):
    sizes, graphs, cross_t, E = gold["sizes"], gold["graphs"], gold["cross_t"], int(gold["e"])
    P, n = len(sizes), int(sizes.sum())
    rng = np.random.default_rng(3)
    cell_of = rng.permutation(np.repeat(np.arange(P, dtype=np.uint32), sizes))  # cells of global ids
    order = np.argsort(cell_of, kind="stable")    # position -> global id (cell order, then id)
    cross_pos = np.ascontiguousarray(cross_t.transpose(1, 0, 2)).reshape(n, P * E)
    cross = np.empty_like(cross_pos)
    cross[order] = cross_pos                      # reference layout: rows in global order
    exp = oracle.expand_spokesman_cross(cell_of, graphs, cross)
    spk, _, _ = oracle.spokesman(sizes, graphs)
    # the row of the point at position p is the row of the point at position spk[p]
    for p in (0, 17, 701, n - 1):
        assert np.array_equal(exp[order[p]], cross[order[spk[p]]])


def test_bad_sizes_and_truncated_files_are_refused(gold, tmp_path):
    with pytest.raises(gf.GarfieldError):
        gf.spokesman(np.array([5, 5], np.uint32), np.zeros((11, 2), np.uint32))
    path = tmp_path / "bad.extreme"
    path.write_bytes(gold["raw"].tobytes()[:-4])
    with pytest.raises(gf.GarfieldError):
        gf.read_spokesman_graph(path)
