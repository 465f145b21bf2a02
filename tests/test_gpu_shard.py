"""GPU parity of cell-sharded search: shard indexes (gf_index_desc.shard_cells) searched
with gf_search_keys and merged with gf_merge_keys equal the oracle's batched search with
the shards as batches.  All shards live on one GPU here; the exchange between ranks is
covered by the gloo test in test_multirank.py."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
from garfield_b200.dist import shard_cells
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def make(c, **kw):
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                           **kw)


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def _oracle(c, batches, **kw):
    ent = c.entry(c.ix.degree)
    return oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                         c.cells, ent, batches=batches, **kw)


@pytest.mark.parametrize("which,world", [("small", 2), ("small", 4), ("odd", 3), ("odd", 8)])
def test_sharded_search_matches_oracle(which, world, request):
    c = request.getfixturevalue(which)
    shards = shard_cells(c.ix.grid, world)
    idx = [make(c, keep_fp32=False, shard_cells=s) for s in shards]
    whole = make(c, keep_fp32=False)
    assert all(i.device_bytes < whole.device_bytes for i in idx) or world == 1
    from conftest import check_shard_plan
    for L, width in ((32, 1), (64, 4)):
        params = gf.SearchParams(L=L, k=10, width=width)
        keys = []
        for i, sh in zip(idx, shards):
            plan = i.plan(c.ds.queries.shape[0])
            plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
            if L == 32:  # each shard orders the cells of its multi-cell queries only
                _, _, cells, top4, _ = plan.read()
                check_shard_plan(c, sh, top4, cells)
            keys.append(plan.search_keys(params).clone())
        ids, dist = idx[0].merge_keys(torch.stack(keys, 0), 10)
        ref_ids, ref_d, _ = _oracle(c, shards, L=L, K=10, width=width)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_ids)
        assert np.array_equal(dist.cpu().numpy(), ref_d)
    # plain search on one shard = the batched oracle restricted to its cells
    plan = idx[-1].plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    ids, dist = plan.search(gf.SearchParams(L=48, k=10))
    ref_ids, ref_d, _ = _oracle(c, [shards[-1]], L=48, K=10)
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), ref_ids)
    assert np.array_equal(dist.cpu().numpy(), ref_d)


def test_keys_of_whole_index_merge_to_plain_search(small):
    c = small
    g = make(c, keep_fp32=False)
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    params = gf.SearchParams(L=40, k=10, width=2)
    ids0, d0 = plan.search(params)
    keys = plan.search_keys(params)
    ids1, d1 = g.merge_keys(keys[None], 10)
    assert torch.equal(ids0, ids1) and torch.equal(d0, d1)
    # keys are sorted and their distance bits are the distances
    k = keys.cpu().numpy().view(np.uint64)
    assert (np.diff(k.astype(np.float64), axis=1) >= 0).all()
    bits = (k >> np.uint64(32)).astype(np.uint32).view(np.float32)
    ok = k != np.uint64(0xFFFFFFFFFFFFFFFF)
    assert np.array_equal(bits[ok], d0.cpu().numpy()[ok])


def test_shard_argument_errors(small):
    c = small
    with pytest.raises(gf.GarfieldError):
        make(c, keep_fp32=False, host_graph=True, shard_cells=[0, 1])
    with pytest.raises(gf.GarfieldError):
        make(c, keep_fp32=False, shard_cells=[0, 0])
    with pytest.raises(gf.GarfieldError):
        make(c, keep_fp32=False, shard_cells=[c.ncells])
    s = make(c, keep_fp32=False, shard_cells=[0, 1])
    plan = s.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    with pytest.raises(gf.GarfieldError) as e:
        plan.search_batched([[0]], gf.SearchParams(L=32))
    assert e.value.status == 7
