"""GPU parity on the shapes of benchmark configurations 3, 4 and 5, drawn at a size the
oracle finishes in seconds (the generators are the full-size ones with fewer points):

- config 3: 96-dim unit-normalised mixture, three attributes (uniform, Zipf(1.1), the
  mixture component's band) on a 4x4x4 grid, ~5% boxes in rank space, k = 100;
- config 4: 768-dim unit-normalised mixture, attributes on [0, 2^20) on an 8x8 grid,
  degree 64, ~2% boxes;
- config 5: uint8 rows (codec 2), a 16x16 grid, ~1% boxes; plain, spokesman-compressed
  (also searched by batches, resident and streamed), scheduled out-of-core batches and four
  cell shards.

Every search compares ids, canonical distances and traversal counters with the oracle bit
for bit; the brute force compares ids and distances with the oracle's exact scan."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

import garfield_b200 as gf
import oracle
from conftest import Case
from garfield_b200 import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def u32(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.fixture(scope="module")
def c3():
    ds = synth.config3(seed=31, n=40000, qnum=300, n_centers=40)
    return Case(0, 0, 0, 0, (), 0, R=32, E=2, C=64, seed=31, ds=ds, k=100, device="cuda")


@pytest.fixture(scope="module")
def c4():
    ds = synth.config4(seed=41, n=12000, qnum=200, n_centers=32)
    return Case(0, 0, 0, 0, (), 0, R=64, E=2, C=32, seed=41, ds=ds, k=10, device="cuda")


@pytest.fixture(scope="module")
def c5():
    ds, codes = synth.config5(seed=51, n=32000, qnum=200, n_centers=32)
    c = Case(0, 0, 0, 0, (), 0, R=32, E=2, C=32, seed=51, ds=ds, k=10, device="cuda")
    c.codes = codes
    return c


def make(c, ix=None, **kw):
    ix = ix or c.ix
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=ix.grid,
                           l_quant=ix.l_quant, r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs,
                           degree=ix.degree, cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, **kw)


def plan_of(g, c):
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    return plan


def ref_search(c, ix=None, **kw):
    return oracle.search(ix or c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts,
                         c.offsets, c.cells, c.entry(c.ix.degree), **kw)


def check_search(c, plan, L, width, k, ix=None, **okw):
    ids, dist = plan.search(gf.SearchParams(L=L, k=k, width=width))
    st = plan.stats()
    ref_ids, ref_d, ref_st = ref_search(c, ix, L=L, K=k, width=width, **okw)
    got = u32(ids)
    assert np.array_equal(got, ref_ids), np.argwhere(got != ref_ids)[:5]
    assert np.array_equal(dist.cpu().numpy(), ref_d)
    assert [st["n_exp"], st["n_cross"], st["n_hops"]] == [int(x) for x in ref_st[1:]]
    return got


def check_filter(c, ids):
    for q in range(ids.shape[0]):
        row = ids[q][ids[q] != gf.NO_ID]
        a = c.ds.attrs[row]
        assert ((a >= c.ds.lo[q]) & (a <= c.ds.hi[q])).all()


def check_bruteforce(c, g, k):
    st = torch.zeros(3, dtype=torch.int32, device="cuda")
    ids, dist = g.bruteforce(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi), k, stats=st)
    assert np.array_equal(u32(ids), c.gt) and np.array_equal(dist.cpu().numpy(), c.gt_d)
    return st.cpu().numpy()


def test_config3_shape(c3):
    c = c3
    assert c.ds.attrs.shape[1] == 3 and c.ncells == 64 and c.ds.vectors.shape[1] == 96
    box = oracle.count_in_box(c.ds.attrs, c.ds.lo, c.ds.hi) / c.ds.vectors.shape[0]
    assert 0.03 < box.mean() < 0.08
    g = make(c, keep_fp32=True)
    plan = plan_of(g, c)
    check_search(c, plan, 256, 4, 100)
    ids = check_search(c, plan, 1024, 8, 100)
    check_filter(c, ids)
    assert oracle.recall(ids, c.gt) >= 0.97
    st = check_bruteforce(c, g, 100)
    assert st[2] > 0 and st[0] <= 0.05 * c.ds.queries.shape[0]  # deep lists on the tensor cores
    plan.close()
    g.close()


def test_config4_shape(c4):
    c = c4
    assert c.ds.vectors.shape[1] == 768 and c.ncells == 64 and c.ix.degree == 64
    g = make(c, keep_fp32=True)
    plan = plan_of(g, c)
    check_search(c, plan, 32, 1, 10)
    ids = check_search(c, plan, 64, 2, 10)
    check_filter(c, ids)
    assert oracle.recall(ids, c.gt) >= 0.98
    st = check_bruteforce(c, g, 10)
    assert st[2] > 0 and st[0] <= 0.05 * c.ds.queries.shape[0]  # tensor-core pass, proven on the device
    plan.close()
    g.close()


def test_config5_shape(c5):
    c = c5
    assert c.ncells == 256 and c.codes.dtype == np.uint8
    dim = c.ds.vectors.shape[1]
    sc = np.full(dim, 0.01, np.float32)
    zp = np.zeros(dim, np.int32)
    okw = dict(alpha=0.01, codec=2, codes=c.codes, scales=sc, zero_points=zp)
    # uint8 rows decode as u / 100 and queries are scaled by 0.01 (f2h_factor)
    g = make(c, keep_fp32=False, codec=2, codes=c.codes, f2h_factor=0.01)
    plan = plan_of(g, c)
    check_search(c, plan, 32, 1, 10, **okw)
    ids = check_search(c, plan, 64, 2, 10, **okw)
    check_filter(c, ids)
    assert oracle.recall(ids, c.gt) >= 0.97
    # out-of-core: batches of at most 16 cells from the device scheduler, rows streamed
    # from pinned host memory
    batches, _ = plan.schedule(16)
    assert all(len(b) <= 16 for b in batches)
    assert set(int(x) for x in c.cells) <= set(x for b in batches for x in b)
    gh = make(c, keep_fp32=False, codec=2, codes=c.codes, f2h_factor=0.01, host_graph=True)
    ph = plan_of(gh, c)
    ids, dist = ph.search_batched(batches, gf.SearchParams(L=48, k=10))
    ref_ids, ref_d, _ = ref_search(c, L=48, K=10, batches=batches, **okw)
    assert np.array_equal(u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    ph.close()
    gh.close()
    # spokesman-compressed cross edges
    gs = make(c, keep_fp32=False, codec=2, codes=c.codes, f2h_factor=0.01, cross_spokesman=True)
    assert gs.cross_rows < c.ds.vectors.shape[0]
    ix2 = dataclasses.replace(c.ix, cross=oracle.expand_spokesman_cross(c.ix.cell_of, c.ix.graphs, c.ix.cross))
    ps = plan_of(gs, c)
    check_search(c, ps, 64, 2, 10, ix=ix2, **okw)
    # the same compressed rows searched by batches, device-resident and streamed from pinned
    # host memory (each batch copies the spokesmen's cross blocks only)
    ref_ids, ref_d, _ = ref_search(c, ix=ix2, L=48, K=10, batches=batches, **okw)
    ids, dist = ps.search_batched(batches, gf.SearchParams(L=48, k=10))
    assert np.array_equal(u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    ghs = make(c, keep_fp32=False, codec=2, codes=c.codes, f2h_factor=0.01, host_graph=True, cross_spokesman=True)
    assert ghs.cross_rows == gs.cross_rows
    phs = plan_of(ghs, c)
    ids, dist = phs.search_batched(batches, gf.SearchParams(L=48, k=10))
    assert np.array_equal(u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    phs.close()
    ghs.close()
    ps.close()
    gs.close()
    # four cell shards, keys merged
    from garfield_b200.dist import shard_cells
    shards = shard_cells(c.ix.grid, 4)
    keys = []
    for s in shards:
        sh = make(c, keep_fp32=False, codec=2, codes=c.codes, f2h_factor=0.01, shard_cells=s)
        p = plan_of(sh, c)
        keys.append(p.search_keys(gf.SearchParams(L=48, k=10)).clone())
        p.close()
    ids, dist = sh.merge_keys(torch.stack(keys, 0), 10)
    ref_ids, ref_d, _ = ref_search(c, L=48, K=10, batches=shards, **okw)
    assert np.array_equal(u32(ids), ref_ids) and np.array_equal(dist.cpu().numpy(), ref_d)
    sh.close()
    # exact scan over the uint8 values
    gb = make(c, keep_fp32=True)
    check_bruteforce(c, gb, 10)
    plan.close()
    g.close()
    gb.close()
