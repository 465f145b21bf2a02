"""Cell-batch scheduler (gf_schedule_batches_host): host logic, runs on CPU."""
from __future__ import annotations

import numpy as np

import garfield_b200 as gf


def _splits(batches, counts, offsets, cells):
    b_of = {c: b for b, cl in enumerate(batches) for c in cl}
    return sum(len({b_of[c] for c in cells[o:o + n]}) for n, o in zip(counts, offsets))


def _grid_plan(side: int, qnum: int, seed: int):
    """Cell lists of random rectangular boxes on a side x side grid (row-major cell ids)."""
    rng = np.random.default_rng(seed)
    lists = []
    for _ in range(qnum):
        w, h = rng.integers(1, 4, size=2)
        x, y = rng.integers(0, side - w + 1), rng.integers(0, side - h + 1)
        lists.append([(y + j) * side + (x + i) for j in range(h) for i in range(w)])
    counts = np.array([len(cl) for cl in lists], np.uint32)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.uint32)
    return counts, offsets, np.concatenate(lists).astype(np.uint32)


def test_schedule_covers_visited_cells_once(small):
    c = small
    for mc in (1, 2, 3, c.ncells, 100):
        batches, splits = gf.schedule_batches(c.ncells, c.counts, c.offsets, c.cells, mc)
        flat = [x for b in batches for x in b]
        visited = set(np.unique(c.cells).tolist())
        assert sorted(flat) == sorted(visited) and len(flat) == len(set(flat))
        assert all(1 <= len(b) <= mc for b in batches)
        assert splits == _splits(batches, c.counts, c.offsets, c.cells)
    batches, splits = gf.schedule_batches(c.ncells, c.counts, c.offsets, c.cells, c.ncells)
    assert len(batches) == 1 and splits == int((c.counts > 0).sum())


def test_schedule_beats_random_partition():
    side = 8
    counts, offsets, cells = _grid_plan(side, 4000, seed=3)
    for mc in (4, 8, 16):
        batches, splits = gf.schedule_batches(side * side, counts, offsets, cells, mc)
        assert splits == _splits(batches, counts, offsets, cells)
        rng = np.random.default_rng(0)
        rand = []
        for _ in range(20):
            perm = rng.permutation(side * side).tolist()
            rand.append(_splits([perm[i:i + mc] for i in range(0, len(perm), mc)], counts, offsets, cells))
        assert splits < min(rand), (mc, splits, min(rand))


def test_schedule_edge_cases():
    empty = np.zeros(0, np.uint32)
    batches, splits = gf.schedule_batches(16, empty, empty, empty, 4)
    assert batches == [] and splits == 0
    counts = np.array([0, 2, 1], np.uint32)
    offsets = np.array([0, 0, 2], np.uint32)
    cells = np.array([5, 3, 5], np.uint32)
    batches, splits = gf.schedule_batches(8, counts, offsets, cells, 1)
    assert batches == [[5], [3]] and splits == 3
    try:
        gf.schedule_batches(8, counts, offsets, cells, 0)
        raise AssertionError("max_cells 0 accepted")
    except gf.GarfieldError as e:
        assert e.status == 1
    try:
        gf.schedule_batches(4, counts, offsets, cells, 2)
        raise AssertionError("cell id >= ncells accepted")
    except gf.GarfieldError as e:
        assert e.status == 1
