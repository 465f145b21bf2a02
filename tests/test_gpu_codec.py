"""GPU parity of the byte codecs (row a18): the device int8 quantiser against the
reference's own .q output, and searches over int8 and uint8 rows against the oracle's
orc_dist8 restatement (ids and distances bit for bit)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GOLDEN = Path(__file__).resolve().parent / "golden"


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def make(c, **kw):
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels, **kw)


def _oracle(c, **kw):
    ent = c.entry(c.ix.degree)
    return oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                         c.cells, ent, **kw)


def test_device_quantiser_matches_reference():
    z = np.load(GOLDEN / "golden_quant.npz")
    x = dev(z["data"])
    for name in ("a1", "a05", "a3"):
        q, sc, zp = gf.quantize_i8(x, float(z[f"{name}_alpha"]))
        assert np.array_equal(q.cpu().numpy(), z[f"{name}_codes"])
        assert np.array_equal(sc.cpu().numpy(), z[f"{name}_scales"])
        assert np.array_equal(zp.cpu().numpy(), z[f"{name}_zps"])


def _search(g, c, params):
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search(params)
    return ids.cpu().numpy().view(np.uint32), dist.cpu().numpy(), plan.stats()


@pytest.mark.parametrize("which", ["small", "odd"])
@pytest.mark.parametrize("alpha", [1.0, 0.5])
def test_int8_search_matches_oracle(which, alpha, request):
    c = request.getfixturevalue(which)
    g = make(c, keep_fp32=False, codec=1, f2h_factor=alpha)  # quantised inside gf_index_create
    q, sc, zp = oracle.quantize_i8(c.ds.vectors, alpha)
    for L, width in ((32, 1), (64, 4)):
        ids, dist, st = _search(g, c, gf.SearchParams(L=L, k=10, width=width))
        ref_ids, ref_d, ref_st = _oracle(c, L=L, K=10, width=width, alpha=alpha, codec=1, codes=q, scales=sc,
                                         zero_points=zp)
        assert np.array_equal(ids, ref_ids)
        assert np.array_equal(dist, ref_d)
        assert [st["n_exp"], st["n_cross"], st["n_hops"]] == [int(x) for x in ref_st[1:]]
    assert oracle.recall(ids, c.gt) >= 0.9
    # exact route over int8 rows
    ids, dist, _ = _search(g, c, gf.SearchParams(L=16, k=10, postfilter=1))
    ref_ids, ref_d, _ = _oracle(c, L=16, K=10, postfilter=1, alpha=alpha, codec=1, codes=q, scales=sc,
                                zero_points=zp)
    assert np.array_equal(ids, ref_ids) and np.array_equal(dist, ref_d)


@pytest.mark.parametrize("which", ["small", "odd"])
def test_uint8_search_matches_oracle(which, request):
    c = request.getfixturevalue(which)
    u8 = np.clip(np.round(c.ds.vectors), 0, 255).astype(np.uint8)
    g = make(c, keep_fp32=False, codec=2, codes=u8, f2h_factor=0.01)  # rows decode u / 100, queries * 0.01
    ids, dist, _ = _search(g, c, gf.SearchParams(L=48, k=10, width=2))
    sc = np.full(c.ds.vectors.shape[1], 0.01, np.float32)
    zp = np.zeros(c.ds.vectors.shape[1], np.int32)
    ref_ids, ref_d, _ = _oracle(c, L=48, K=10, width=2, alpha=0.01, codec=2, codes=u8, scales=sc, zero_points=zp)
    assert np.array_equal(ids, ref_ids) and np.array_equal(dist, ref_d)
    assert oracle.recall(ids, c.gt) >= 0.75  # integer rounding of the vectors costs recall


def test_codec_with_batches_and_shards(small):
    """The byte codec composes with the batched, host-streamed and sharded searches."""
    from garfield_b200.dist import shard_cells
    c = small
    q, sc, zp = gf.quantize_i8_host(c.ds.vectors, 1.0)
    batches = [[0, 3], [1, 2]]
    ref_ids, ref_d, _ = _oracle(c, L=40, K=10, codec=1, codes=q, scales=sc, zero_points=zp, batches=batches)
    g = make(c, keep_fp32=False, codec=1, codes=q, code_scales=sc, code_zero_points=zp, host_graph=True)
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search_batched(batches, gf.SearchParams(L=40, k=10))
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_ids)
    assert np.array_equal(dist.cpu().numpy(), ref_d)
    shards = shard_cells(c.ix.grid, 2)
    keys = []
    for s in shards:
        sh = make(c, keep_fp32=False, codec=1, codes=q, code_scales=sc, code_zero_points=zp, shard_cells=s)
        p = sh.plan(c.ds.queries.shape[0])
        p.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
        keys.append(p.search_keys(gf.SearchParams(L=40, k=10)).clone())
    ids, dist = sh.merge_keys(torch.stack(keys, 0), 10)
    ref_ids, ref_d, _ = _oracle(c, L=40, K=10, codec=1, codes=q, scales=sc, zero_points=zp, batches=shards)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_ids)
    assert np.array_equal(dist.cpu().numpy(), ref_d)


def test_open_with_q_file_and_u8bin(small, tmp_path):
    """gf_index_open with a .q file (codec 1) and with u8bin data (codec 2)."""
    c = small
    from garfield_b200 import indexbuild
    paths = indexbuild.write_files(tmp_path, "t", c.ds, c.ix)
    files = {k: paths[k] for k in ("data_path", "cagra_prefix", "cagra_suffix", "global_graph", "grid", "attrs",
                                   "cluster")}
    files["degree"] = c.ix.degree
    q, sc, zp = gf.quantize_i8_host(c.ds.vectors, 1.0)
    gf.write_q(tmp_path / "data.q", q, sc, zp)
    g = gf.Index.open(**files, codec=1, quantized=tmp_path / "data.q")
    ids, dist, _ = _search(g, c, gf.SearchParams(L=40, k=10))
    ref_ids, ref_d, _ = _oracle(c, L=40, K=10, codec=1, codes=q, scales=sc, zero_points=zp)
    assert np.array_equal(ids, ref_ids) and np.array_equal(dist, ref_d)
    u8 = np.clip(np.round(c.ds.vectors), 0, 255).astype(np.uint8)
    with open(tmp_path / "data.u8bin", "wb") as f:
        f.write(np.array(u8.shape, np.uint32).tobytes() + u8.tobytes())
    files["data_path"] = tmp_path / "data.u8bin"
    g = gf.Index.open(**files, codec=2, f2h_factor=0.01)  # the query scaled like the rows (u / 100)
    ids, dist, _ = _search(g, c, gf.SearchParams(L=40, k=10))
    sc8 = np.full(u8.shape[1], 0.01, np.float32)
    # the planner's centroids now come from the u8 rows: order the cells the same way
    cent, hist = oracle.cluster_info(u8.astype(np.float32), c.ix.labels, c.ix.cell_of, c.ncells)
    cells, _ = oracle.order_cells(c.ds.queries, cent, hist, c.counts, c.offsets, c.cells_unordered)
    ent = c.entry(c.ix.degree)
    ref_ids, ref_d, _ = oracle.search(c.ix, u8.astype(np.float32), c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi,
                                      c.counts, c.offsets, cells, ent, L=40, K=10, alpha=0.01, codec=2, codes=u8,
                                      scales=sc8, zero_points=np.zeros(u8.shape[1], np.int32))
    assert np.array_equal(ids, ref_ids) and np.array_equal(dist, ref_d)
