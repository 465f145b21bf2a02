"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def _cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


class Case:
    """A small synthetic dataset with its index (reference layout) and oracle plan."""

    def __init__(self, n, dim, centers, qnum, grid, sel, R, E, C, seed, sigma=20.0, stratified=True, domain=10000,
                 ds=None, k=10, device="cpu"):
        from garfield_b200 import indexbuild, synth
        import oracle
        if ds is None:
            ds = synth.make(n, dim, centers, qnum, grid, sel, domain=domain, sigma=sigma, seed=seed,
                            stratified=stratified)
        self.ds = ds
        grid = tuple(ds.grid)
        self.ix = indexbuild.build(self.ds.vectors, self.ds.attrs, grid, R=R, E=E, C=C, seed=seed, device=device)
        self.grid = grid
        self.ncells = int(np.prod(grid))
        self.counts, self.offsets, self.cells_unordered = oracle.plan_cells(self.ds.lo, self.ds.hi, self.ix.grid,
                                                                           self.ix.l_quant, self.ix.r_quant)
        self.centroids, self.hist = oracle.cluster_info(self.ds.vectors, self.ix.labels, self.ix.cell_of, self.ncells)
        self.cells, self.top4 = oracle.order_cells(self.ds.queries, self.centroids, self.hist, self.counts,
                                                   self.offsets, self.cells_unordered)
        self.k = k
        self.gt, self.gt_d = oracle.bruteforce(self.ds.vectors, self.ds.attrs, self.ds.queries, self.ds.lo,
                                               self.ds.hi, k)

    def entry(self, n):
        """The library's entry sequence: std::mt19937 default seed, draw % range, distinct."""
        return mt_entry(n, int(np.bincount(self.ix.cell_of, minlength=self.ncells).min()))


def mt19937_stream():
    """Python's random.Random(5489) is not std::mt19937's seeding; restate the engine."""
    mt = [0] * 624
    mt[0] = 5489
    for i in range(1, 624):
        mt[i] = (1812433253 * (mt[i - 1] ^ (mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
    idx = 624
    while True:
        if idx >= 624:
            for i in range(624):
                y = (mt[i] & 0x80000000) | (mt[(i + 1) % 624] & 0x7FFFFFFF)
                mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ (0x9908B0DF if y & 1 else 0)
            idx = 0
        y = mt[idx]
        idx += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        yield y


def mt_entry(n: int, rng_range: int) -> np.ndarray:
    out, seen = [], set()
    n = min(n, rng_range)
    for v in mt19937_stream():
        t = v % rng_range
        if t not in seen:
            seen.add(t)
            out.append(t)
            if len(out) == n:
                break
    return np.array(out, np.uint32)


@pytest.fixture(scope="session")
def small():
    """20k x 64, 2x2 grid, R=16."""
    return Case(20000, 64, 50, 300, (2, 2), 0.10, R=16, E=2, C=50, seed=11)


@pytest.fixture(scope="session")
def odd():
    """12k x 100 (row padding), 3 attributes on a 2x2x2 grid, unbalanced quantile cells."""
    return Case(12000, 100, 40, 200, (2, 2, 2), 0.15, R=16, E=2, C=40, seed=23, stratified=False)


def check_shard_plan(c, shard, top4, cells):
    """A shard's plan (gf_plan_read of a shard_cells index) against the whole-index plan
    c.top4 / c.cells: queries with two or more of the shard's cells get the same top4 and
    cell order; the others keep top4 empty and their cells in increasing id."""
    held = set(int(x) for x in shard)
    n_local = 0
    for q in range(c.counts.shape[0]):
        o, m = int(c.offsets[q]), int(c.counts[q])
        mine = cells[o:o + m]
        if sum(int(x) in held for x in mine) >= 2:
            n_local += 1
            assert np.array_equal(top4[q], c.top4[q]), q
            assert np.array_equal(mine, c.cells[o:o + m]), q
        else:
            assert (top4[q] == 0xFFFFFFFF).all(), q
            assert np.array_equal(mine, np.sort(c.cells[o:o + m])), q
    return n_local
