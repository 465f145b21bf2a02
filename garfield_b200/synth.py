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
         normalize: bool = False, center_hi: float = 255.0, sphere: bool = False) -> Dataset:
    rv = np.random.default_rng(seed)
    if sphere:
        vectors, centers, labels = sphere_mixture(n, dim, n_centers, sigma, rv)
    else:
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
                        sigma=sigma, seed=seed, normalize=normalize, sphere=sphere, center_hi=center_hi))


def sphere_mixture(n: int, dim: int, n_centers: int, sigma: float, rng: np.random.Generator,
                   centers: np.ndarray | None = None, chunk: int = 1 << 18):
    """Unit-normalised mixture: centers are N(0, 1)^dim directions scaled to norm 1, a point
    is its center plus N(0, sigma^2) noise per coordinate, normalised to norm 1 afterwards."""
    if centers is None:
        centers = rng.standard_normal((n_centers, dim), dtype=np.float32)
        centers /= np.maximum(np.linalg.norm(centers, axis=1, keepdims=True), 1e-12)
    return gaussian_mixture(n, dim, centers.shape[0], sigma, rng, centers=centers, clip_min=None,
                            normalize=True, chunk=chunk)


def zipf_attr(n: int, domain: int, s: float, rng: np.random.Generator) -> np.ndarray:
    """Bounded Zipf on [0, domain): P(v) proportional to (v + 1)^-s, by inverse CDF."""
    w = np.arange(1, domain + 1, dtype=np.float64) ** -s
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    v = np.searchsorted(cdf, rng.random(n), side="right")
    return np.minimum(v, domain - 1).astype(np.int32)


def cluster_attr(labels: np.ndarray, n_centers: int, domain: int, rng: np.random.Generator) -> np.ndarray:
    """An attribute correlated with the mixture component: a uniform integer inside the
    component's own band [label, label + 1) * domain / n_centers."""
    u = rng.random(labels.shape[0])
    return np.minimum(np.floor((labels + u) * (domain / n_centers)), domain - 1).astype(np.int32)


def quantile_boxes(attrs: np.ndarray, qnum: int, selectivity: float, rng: np.random.Generator):
    """Closed boxes drawn in rank space: in every dimension the side spans
    selectivity^(1/a) of the points (by rank), placed uniformly; bounds are the attribute
    values at the two end ranks.  On skewed attributes (Zipf) ties widen a side, so the
    selectivity is approximate."""
    n, a = attrs.shape
    side = max(1, min(n, int(round(n * selectivity ** (1.0 / a)))))
    lo = np.empty((qnum, a), np.int32)
    hi = np.empty((qnum, a), np.int32)
    for j in range(a):
        srt = np.sort(attrs[:, j])
        st = rng.integers(0, n - side + 1, size=qnum)
        lo[:, j] = srt[st]
        hi[:, j] = srt[st + side - 1]
    return lo, hi


# Benchmark configurations (BASELINE.json configs[0] .. configs[4]).  Configs 3-5 take the
# point count, query count and center count as arguments so that tests can draw the same
# distributions at a size the oracle finishes in seconds.
def config1(seed: int = DEFAULT_SEED, n: int = 100_000, qnum: int = 1000) -> Dataset:
    """100k x 128, 100-center mixture, 2 uniform attributes, 1000 queries, ~10% boxes."""
    return make(n, 128, 100, qnum, (4, 4), 0.10, seed=seed, stratified=False)


def config2(seed: int = DEFAULT_SEED, selectivity: float = 0.10, n: int = 1_000_000, qnum: int = 10_000) -> Dataset:
    """1M x 128, 1000-center mixture, 2 attributes on a 4x4 grid, 10k queries."""
    return make(n, 128, 1000, qnum, (4, 4), selectivity, seed=seed, stratified=True)


def config3(seed: int = DEFAULT_SEED, n: int = 10_000_000, qnum: int = 100_000, n_centers: int = 10_000,
            selectivity: float = 0.05) -> Dataset:
    """10M x 96 unit-normalised mixture (sigma 0.1 per coordinate before normalisation);
    attributes U[0, 10000), Zipf(1.1) on [0, 10000) and the component's band; 4x4x4 grid;
    100k queries from the mixture with rank-space 3-D boxes of ~5% selectivity."""
    domain = 10000
    rv = np.random.default_rng(seed)
    vectors, centers, labels = sphere_mixture(n, 96, n_centers, 0.1, rv)
    ra = np.random.default_rng(seed + 1)
    attrs = np.stack([ra.integers(0, domain, size=n, dtype=np.int64).astype(np.int32),
                      zipf_attr(n, domain, 1.1, ra), cluster_attr(labels, n_centers, domain, ra)], 1)
    rq = np.random.default_rng(seed + 2)
    queries, _, _ = sphere_mixture(qnum, 96, n_centers, 0.1, rq, centers=centers)
    lo, hi = quantile_boxes(attrs, qnum, selectivity, np.random.default_rng(seed + 3))
    return Dataset(vectors, attrs, queries, lo, hi, (4, 4, 4), None,
                   dict(n=n, dim=96, n_centers=n_centers, qnum=qnum, selectivity=selectivity, domain=domain,
                        sigma=0.1, seed=seed, k=100, R=32, E=0))


def config4(seed: int = DEFAULT_SEED, n: int = 1_000_000, qnum: int = 10_000, n_centers: int = 2000,
            selectivity: float = 0.02, sigma: float = 0.02) -> Dataset:
    """1M x 768 unit-normalised embedding-like mixture (sigma 0.02 per coordinate: noise of
    norm ~0.55 around unit centers); 2 attributes U[0, 2^20) on an 8x8 grid; 10k queries
    with ~2% boxes."""
    return make(n, 768, n_centers, qnum, (8, 8), selectivity, domain=1 << 20, sigma=sigma, seed=seed,
                stratified=False, normalize=True, sphere=True)


def config5(seed: int = DEFAULT_SEED, n: int = 1_000_000_000, qnum: int = 100_000, n_centers: int = 100_000,
            selectivity: float = 0.01):
    """1B x 128 uint8 (the config-1 mixture rounded and clipped to [0, 255]); 2 attributes
    U[0, 10000) on a 16x16 grid; 100k queries with ~1% boxes.  Returns the Dataset (fp32
    vectors) and the uint8 rows."""
    ds = make(n, 128, n_centers, qnum, (16, 16), selectivity, seed=seed, stratified=True)
    codes = np.clip(np.rint(ds.vectors), 0, 255).astype(np.uint8)
    ds.vectors = codes.astype(np.float32)
    ds.meta.update(k=10, R=32, E=2)
    return ds, codes


def query_stream(ds: Dataset, stream: int, selectivity: float | None = None) -> Dataset:
    """Another batch of queries from `ds`'s distribution (same mixture centers, same box
    rule, the same number of queries) for the query stream `stream` >= 1 of a multi-GPU
    run; stream 0 is ds itself.  The centers are redrawn from the vector seed (they are
    the first draw of its generator); queries and boxes use seeds seed + 2 + 1000 * stream
    and seed + 3 + 1000 * stream.  Only for make()-style datasets (configs 1, 2, 4, 5)."""
    if stream == 0:
        return ds
    m = ds.meta
    seed, dim, n_centers, qnum = m["seed"], m["dim"], m["n_centers"], m["qnum"]
    sel = m["selectivity"] if selectivity is None else selectivity
    normalize = bool(m.get("normalize", False))
    sphere = bool(m.get("sphere", False))
    rv = np.random.default_rng(seed)
    if sphere:
        centers = rv.standard_normal((n_centers, dim), dtype=np.float32)
        centers /= np.maximum(np.linalg.norm(centers, axis=1, keepdims=True), 1e-12)
    else:
        centers = rv.uniform(0.0, m.get("center_hi", 255.0), size=(n_centers, dim)).astype(np.float32)
    rq = np.random.default_rng(seed + 2 + 1000 * stream)
    if sphere:
        queries, _, _ = sphere_mixture(qnum, dim, n_centers, m["sigma"], rq, centers=centers)
    else:
        queries, _, _ = gaussian_mixture(qnum, dim, n_centers, m["sigma"], rq, centers=centers,
                                         clip_min=None if normalize else 0.0, normalize=normalize)
    rb = np.random.default_rng(seed + 3 + 1000 * stream)
    lo, hi = boxes(qnum, len(ds.grid), m["domain"], sel, rb)
    return Dataset(ds.vectors, ds.attrs, queries, lo, hi, ds.grid, ds.cell_of, dict(m, stream=stream))
