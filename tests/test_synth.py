"""The seeded generators of configurations 3-5 (CPU): shapes, value ranges and the
distributions each configuration names, drawn at a reduced size."""
from __future__ import annotations

import numpy as np

from garfield_b200 import synth


def test_config3_distributions():
    ds = synth.config3(seed=5, n=60000, qnum=400, n_centers=50)
    n = ds.vectors.shape[0]
    assert ds.vectors.shape == (60000, 96) and ds.queries.shape == (400, 96) and ds.grid == (4, 4, 4)
    assert np.allclose(np.linalg.norm(ds.vectors, axis=1), 1.0, atol=1e-5)
    assert np.allclose(np.linalg.norm(ds.queries, axis=1), 1.0, atol=1e-5)
    a = ds.attrs
    assert a.dtype == np.int32 and a.min() >= 0 and a.max() < 10000
    # uniform, Zipf(1.1) (value 0 most frequent, P(0) = 1 / H(10000, 1.1)), component band
    assert abs(np.mean(a[:, 0]) - 5000) < 100
    h = np.sum(np.arange(1, 10001, dtype=np.float64) ** -1.1)
    assert abs(np.mean(a[:, 1] == 0) - 1 / h) < 0.01
    assert np.mean(a[:, 1] < 10) > 0.2
    band = 10000 / 50
    # points of one component share one band: the band index repeats within a component
    comp = np.floor(a[:, 2] / band).astype(int)
    assert len(np.unique(comp)) == 50
    sel = ((a[None] >= ds.lo[:, None]) & (a[None] <= ds.hi[:, None])).all(2).mean(1)
    assert 0.03 < sel.mean() < 0.08 and (ds.hi >= ds.lo).all()
    again = synth.config3(seed=5, n=60000, qnum=400, n_centers=50)
    assert np.array_equal(again.vectors, ds.vectors) and np.array_equal(again.lo, ds.lo)


def test_config4_and_5_shapes():
    ds = synth.config4(seed=6, n=5000, qnum=100, n_centers=20)
    assert ds.vectors.shape == (5000, 768) and ds.grid == (8, 8)
    assert np.allclose(np.linalg.norm(ds.vectors, axis=1), 1.0, atol=1e-5)
    assert ds.attrs.max() < (1 << 20) and ds.attrs.max() > (1 << 19)
    sel = ((ds.attrs[None] >= ds.lo[:, None]) & (ds.attrs[None] <= ds.hi[:, None])).all(2).mean(1)
    assert 0.01 < sel.mean() < 0.03
    ds5, codes = synth.config5(seed=7, n=25600, qnum=100, n_centers=20)
    assert codes.dtype == np.uint8 and codes.shape == (25600, 128) and ds5.grid == (16, 16)
    assert np.array_equal(ds5.vectors, codes.astype(np.float32))
    # stratified attributes: every one of the 256 cells holds n / 256 points
    assert np.array_equal(np.bincount(ds5.cell_of, minlength=256), np.full(256, 100))


def test_quantile_boxes_on_ties():
    rng = np.random.default_rng(3)
    attrs = np.stack([np.zeros(1000, np.int32), rng.integers(0, 100, 1000).astype(np.int32)], 1)
    lo, hi = synth.quantile_boxes(attrs, 50, 0.25, np.random.default_rng(4))
    assert (lo[:, 0] == 0).all() and (hi[:, 0] == 0).all()  # a constant attribute: every box holds it
    assert (hi[:, 1] >= lo[:, 1]).all()


def test_query_stream_draws_new_queries_from_the_same_distribution():
    """Multi-GPU weak scaling: rank r searches query stream r (stream 0 = the dataset's own
    batch).  Other streams are reproducible, differ from stream 0 and come from the same
    mixture centers and box rule."""
    from garfield_b200 import synth
    ds = synth.make(4000, 16, 8, 200, (2, 2), 0.10, seed=5)
    assert synth.query_stream(ds, 0) is ds
    s1, s1b, s2 = synth.query_stream(ds, 1), synth.query_stream(ds, 1), synth.query_stream(ds, 2)
    assert np.array_equal(s1.queries, s1b.queries) and np.array_equal(s1.lo, s1b.lo)
    assert not np.array_equal(s1.queries, ds.queries) and not np.array_equal(s1.queries, s2.queries)
    assert s1.queries.shape == ds.queries.shape and s1.queries.dtype == ds.queries.dtype
    assert s1.vectors is ds.vectors and s1.attrs is ds.attrs
    assert np.array_equal(s1.hi - s1.lo, ds.hi - ds.lo)  # same box side
    centers = np.random.default_rng(5).uniform(0.0, 255.0, size=(8, 16)).astype(np.float32)

    def nearest(q):
        return ((q[:, None, :] - centers[None]) ** 2).sum(-1).min(1).mean()
    assert abs(nearest(s1.queries) / nearest(ds.queries) - 1) < 0.1
