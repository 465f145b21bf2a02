"""File formats through the C ABI readers/writers (no GPU): round trips, reference
layouts written independently with numpy, and error reporting on bad files."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf


def test_fvecs_roundtrip(tmp_path):
    x = np.random.default_rng(0).standard_normal((37, 13)).astype(np.float32)
    p = tmp_path / "a.fvecs"
    gf.write_fvecs(p, x)
    raw = np.fromfile(p, dtype=np.int32).reshape(37, 14)  # tools.cuh:85-106 layout
    assert (raw[:, 0] == 13).all()
    assert np.array_equal(raw[:, 1:].view(np.float32), x)
    assert np.array_equal(gf.read_fvecs(p), x)


def test_attrs_roundtrip(tmp_path):
    a = np.random.default_rng(1).integers(-5, 10000, (50, 3)).astype(np.int32)
    p = tmp_path / "x.attrs"
    gf.write_attrs(p, a)
    raw = np.fromfile(p, dtype=np.int32)
    assert raw[0] == 50 and raw[1] == 3 and np.array_equal(raw[2:].reshape(50, 3), a)
    assert np.array_equal(gf.read_attrs(p), a)


def test_u32mat_roundtrip(tmp_path):
    m = np.random.default_rng(2).integers(0, 2**32, (19, 7), dtype=np.uint64).astype(np.uint32)
    p = tmp_path / "g.graph"
    gf.write_u32mat(p, m)
    assert np.array_equal(gf.read_u32mat(p), m)


def test_ranges_interleaved(tmp_path):
    lo = np.array([[1, 2], [3, 4]], np.int32)
    hi = np.array([[10, 20], [30, 40]], np.int32)
    p = tmp_path / "r.range"
    gf.write_ranges(p, lo, hi)
    # tools.cuh:275-291: per query, per attribute (l, r)
    assert np.array_equal(np.fromfile(p, np.int32), np.array([1, 10, 2, 20, 3, 30, 4, 40], np.int32))
    l2, h2 = gf.read_ranges(p, 2, 2)
    assert np.array_equal(l2, lo) and np.array_equal(h2, hi)


def test_labels_and_grid(tmp_path, small):
    from garfield_b200 import indexbuild
    paths = indexbuild.write_files(tmp_path, "t", small.ds, small.ix)
    lab = gf.read_labels(paths["cluster"])
    assert np.array_equal(lab, small.ix.labels)
    grid, lq, rq, cell_of = gf.read_grid(paths["grid"])
    assert np.array_equal(grid, small.ix.grid)
    assert np.array_equal(lq, small.ix.l_quant) and np.array_equal(rq, small.ix.r_quant)
    assert np.array_equal(cell_of, small.ix.cell_of)
    for c in range(small.ncells):
        g = gf.read_u32mat(f"{paths['cagra_prefix']}{c}{paths['cagra_suffix']}")
        assert g.shape == ((small.ix.cell_of == c).sum(), small.ix.degree)
    assert np.array_equal(gf.read_u32mat(paths["global_graph"]), small.ix.cross)


def test_errors(tmp_path):
    with pytest.raises(gf.GarfieldError) as e:
        gf.read_fvecs(tmp_path / "missing.fvecs")
    assert e.value.status == 2  # GF_ERR_IO
    p = tmp_path / "trunc.fvecs"
    np.array([4, 0, 0], np.int32).tofile(p)  # header says 4 floats, only 2 follow
    with pytest.raises(gf.GarfieldError) as e:
        gf.read_fvecs(p)
    assert e.value.status == 3  # GF_ERR_FORMAT
    p = tmp_path / "bad.attrs"
    np.array([10, 2, 1, 2, 3], np.int32).tofile(p)
    with pytest.raises(gf.GarfieldError) as e:
        gf.read_attrs(p)
    assert e.value.status == 3
    p = tmp_path / "bad.grid"
    np.array([5, 1, 2, 0, 1], np.int32).tofile(p)
    with pytest.raises(gf.GarfieldError) as e:
        gf.read_grid(p)
    assert e.value.status == 3


def test_q_file_round_trip(tmp_path):
    rng = np.random.default_rng(4)
    codes = rng.integers(-128, 128, size=(37, 20)).astype(np.int8)
    sc = rng.random(20).astype(np.float32)
    zp = rng.integers(-128, 128, size=20).astype(np.int32)
    gf.write_q(tmp_path / "x.q", codes, sc, zp)
    c2, s2, z2 = gf.read_q(tmp_path / "x.q")
    assert np.array_equal(c2, codes) and np.array_equal(s2, sc) and np.array_equal(z2, zp)
    raw = (tmp_path / "x.q").read_bytes()
    (tmp_path / "bad.q").write_bytes(raw[:-1])
    with pytest.raises(gf.GarfieldError) as e:
        gf.read_q(tmp_path / "bad.q")
    assert e.value.status == 3
