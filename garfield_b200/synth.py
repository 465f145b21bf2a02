"""Seeded synthetic datasets with the shapes of the benchmark configurations.

The reference is measured on SIFT1M / Deep / DBLP / YouTube files that are not
available here; these generators stand in for them with the distributions the
configurations name (Gaussian mixtures, uniform integer attributes, range boxes of a
given selectivity).  numpy's PCG64 generator makes the data identical on every machine.

Seeds: vectors `seed`, attributes `seed + 1`, queries `seed + 2`, boxes `seed + 3`.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

DEFAULT_SEED = 20261201


def gaussian_mixture(n: int, dim: int, n_centers: int, sigma: float, rng: np.random.Generator,
                     centers: np.ndarray | None = None, lo: float = 0.0, hi: float = 255.0,
                     clip_min: float | None = 0.0, normalize: bool = False, chunk: int = 1 << 18):
    """n points around n_centers centers drawn U[lo, hi)^dim (or given), N(0, sigma^2) noise."""
    if centers is None:
        centers = rng.uniform(lo, hi, size=(n_centers, dim)).astype(np.float32)
    labels = rng.integers(0, centers.shape[0], size=n)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        x = centers[labels[s:e]] + rng.standard_normal((e - s, dim), dtype=np.float32) * np.float32(sigma)
        if clip_min is not None:
            np.maximum(x, clip_min, out=x)
        if normalize:
            x /= np.maximum(np.linalg.norm(x, axis=1, keepdims=True), 1e-12)
        out[s:e] = x
    return out, centers, labels


def cell_sizes(n: int, n_cells: int) -> np.ndarray:
    base = np.full(n_cells, n // n_cells, np.int64)
    base[: n % n_cells] += 1
    return base


def stratified_uniform_attrs(n: int, grid: tuple[int, ...], domain: int, rng: np.random.Generator):
    """Integer attributes uniform on [0, domain) per dimension, stratified so that the
    quantile grid of `grid` slices per dimension puts exactly n / prod(grid) points in
    every cell; points are ordered cell by cell (point i lies in cell i // (n/cells)).

    Each dimension's domain is cut into grid[j] equal ranges; a point of cell c takes, in
    dimension j, a uniform integer from the range of its slice index.  The per-dimension
    marginals are uniform on [0, domain); the cells of the quantile grid
    (grid_scatter_V2, indexbuild/tools.py:88-125) are exactly these ranges.
    """
    a = len(grid)
    n_cells = int(np.prod(grid))
    sizes = cell_sizes(n, n_cells)
    cell_of = np.repeat(np.arange(n_cells, dtype=np.uint32), sizes)
    attrs = np.empty((n, a), np.int32)
    rem = cell_of.astype(np.int64)
    idx = np.empty((n, a), np.int64)
    for j in range(a - 1, -1, -1):  # row-major mixed radix, last dimension fastest
        idx[:, j] = rem % grid[j]
        rem //= grid[j]
    for j in range(a):
        w = domain // grid[j]
        base = idx[:, j] * w
        width = np.where(idx[:, j] == grid[j] - 1, domain - base, w)
        attrs[:, j] = (base + np.floor(rng.random(n) * width)).astype(np.int32)
    return attrs, cell_of


def uniform_attrs(n: int, a: int, domain: int, rng: np.random.Generator) -> np.ndarray:
    return rng.integers(0, domain, size=(n, a), dtype=np.int64).astype(np.int32)


def boxes(qnum: int, a: int, domain: int, selectivity: float, rng: np.random.Generator):
    """Axis-aligned closed integer boxes whose volume is `selectivity` of the domain:
    each side covers selectivity^(1/a) of [0, domain), placed uniformly at random."""
    side = max(1, int(round(domain * selectivity ** (1.0 / a))))
    side = min(side, domain)
    lo = rng.integers(0, domain - side + 1, size=(qnum, a), dtype=np.int64)
    return lo.astype(np.int32), (lo + side - 1).astype(np.int32)


@dataclass
class Dataset:
    vectors: np.ndarray
    attrs: np.ndarray            # int32 n x a
    queries: np.ndarray
    lo: np.ndarray               # int32 qnum x a
    hi: np.ndarray
    grid: tuple = ()
    cell_of: np.ndarray | None = None
    meta: dict = field(default_factory=dict)


def make(n: int, dim: int, n_centers: int, qnum: int, grid: tuple[int, ...], selectivity: float,
         domain: int = 10000, sigma: float = 20.0, seed: int = DEFAULT_SEED, stratified: bool = True,
         normalize: bool = False, center_hi: float = 255.0) -> Dataset:
    rv = np.random.default_rng(seed)
    vectors, centers, labels = gaussian_mixture(n, dim, n_centers, sigma, rv, hi=center_hi,
                                                clip_min=None if normalize else 0.0, normalize=normalize)
    ra = np.random.default_rng(seed + 1)
    if stratified:
        attrs, cell_of = stratified_uniform_attrs(n, grid, domain, ra)
    else:
        attrs, cell_of = uniform_attrs(n, len(grid), domain, ra), None
    rq = np.random.default_rng(seed + 2)
    queries, _, qlabels = gaussian_mixture(qnum, dim, n_centers, sigma, rq, centers=centers,
                                           clip_min=None if normalize else 0.0, normalize=normalize)
    rb = np.random.default_rng(seed + 3)
    lo, hi = boxes(qnum, len(grid), domain, selectivity, rb)
    return Dataset(vectors, attrs, queries, lo, hi, tuple(grid), cell_of,
                   dict(n=n, dim=dim, n_centers=n_centers, qnum=qnum, selectivity=selectivity, domain=domain,
                        sigma=sigma, seed=seed))


# Benchmark configurations; configs 3-5 follow
# the same generators with their own shapes.
def config1(seed: int = DEFAULT_SEED, n: int = 100_000, qnum: int = 1000) -> Dataset:
    """100k x 128, 100-center mixture, 2 uniform attributes, 1000 queries, ~10% boxes."""
    return make(n, 128, 100, qnum, (4, 4), 0.10, seed=seed, stratified=False)


def config2(seed: int = DEFAULT_SEED, selectivity: float = 0.10, n: int = 1_000_000, qnum: int = 10_000) -> Dataset:
    """1M x 128, 1000-center mixture, 2 attributes on a 4x4 grid, 10k queries."""
    return make(n, 128, 1000, qnum, (4, 4), selectivity, seed=seed, stratified=True)
