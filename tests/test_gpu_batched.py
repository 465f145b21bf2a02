"""GPU parity of gf_search_batched (search restricted to batches of cells, results merged
over batches) against the oracle's orc_search_batched, for a device-resident index and for
an index whose graphs stay in pinned host memory and are copied per batch."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def make_index(c, host_graph=False):
    return gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                           l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                           degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels,
                           keep_fp32=False, host_graph=host_graph)


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def as_u32(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.fixture(scope="module")
def indexes(small, odd):
    return {(w, h): make_index(c, h) for w, c in (("small", small), ("odd", odd)) for h in (False, True)}


def _plan(g, c):
    plan = g.plan(c.ds.queries.shape[0])
    plan.build(dev(c.ds.queries), dev(c.ds.lo), dev(c.ds.hi))
    return plan


def _oracle(c, batches, **kw):
    ent = c.entry(c.ix.degree)
    return oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                         c.cells, ent, batches=batches, **kw)


def _splits(ncells):
    rng = np.random.default_rng(11)
    perm = rng.permutation(ncells).tolist()
    half = ncells // 2
    return [
        [list(range(ncells))],                                   # one batch: plain search
        [sorted(perm[:half]), sorted(perm[half:])],               # two batches
        [[x] for x in perm],                                      # one cell per batch (turns reused)
        [perm[: half + 1][::-1], perm[half + 1:]],                # unsorted cell lists
    ]


@pytest.mark.parametrize("which", ["small", "odd"])
@pytest.mark.parametrize("host_graph", [False, True])
def test_batched_matches_oracle(which, host_graph, request, indexes):
    c = request.getfixturevalue(which)
    g = indexes[(which, host_graph)]
    plan = _plan(g, c)
    for batches in _splits(c.ncells):
        for L, width in ((32, 1), (64, 4)):
            params = gf.SearchParams(L=L, k=10, width=width)
            ids, dist = plan.search_batched(batches, params)
            st = plan.stats()
            ref_ids, ref_d, ref_st = _oracle(c, batches, L=L, K=10, width=width)
            assert np.array_equal(as_u32(ids), ref_ids), (batches, L, width)
            assert np.array_equal(dist.cpu().numpy(), ref_d)
            # n_dist may exceed the oracle's: the GPU visited hash is a cache that can forget
            assert [st["n_exp"], st["n_cross"], st["n_hops"]] == [int(x) for x in ref_st[1:]]
            assert st["n_dist"] >= int(ref_st[0])


@pytest.mark.parametrize("which", ["small", "odd"])
def test_one_batch_is_plain_search(which, request, indexes):
    c = request.getfixturevalue(which)
    g = indexes[(which, False)]
    plan = _plan(g, c)
    params = gf.SearchParams(L=48, k=10, width=2)
    ids0, d0 = plan.search(params)
    st0 = plan.stats()
    ids1, d1 = plan.search_batched([list(range(c.ncells))], params)
    st1 = plan.stats()
    assert torch.equal(ids0, ids1) and torch.equal(d0, d1)
    assert st0 == st1
    # the host-graph index gives the same result through the copies
    ids2, d2 = _plan(indexes[(which, True)], c).search_batched([list(range(c.ncells))], params)
    assert torch.equal(ids0, ids2) and torch.equal(d0, d2)


def test_exact_route_and_partial_cover(small, indexes):
    c = small
    g = indexes[("small", True)]
    plan = _plan(g, c)
    params = gf.SearchParams(L=16, k=10, postfilter=1)
    ids, _ = plan.search_batched([[x] for x in range(c.ncells)], params)
    ref, _, _ = _oracle(c, None, L=16, K=10, postfilter=1)
    assert np.array_equal(as_u32(ids), ref)
    # cells in no batch contribute nothing
    ids, _ = plan.search_batched([[1]], gf.SearchParams(L=32, k=10))
    ref, _, _ = _oracle(c, [[1]], L=32, K=10)
    got = as_u32(ids)
    assert np.array_equal(got, ref)
    assert np.isin(got, np.append(np.flatnonzero(c.ix.cell_of == 1), gf.NO_ID)).all()
    # no batches at all: every result empty
    ids, dist = plan.search_batched([], gf.SearchParams(L=32, k=10))
    assert (as_u32(ids) == gf.NO_ID).all() and torch.isinf(dist).all()


def test_batched_errors(small, indexes):
    c = small
    g = indexes[("small", True)]
    plan = _plan(g, c)
    with pytest.raises(gf.GarfieldError) as e:
        plan.search_batched([[0, 1], [1]], gf.SearchParams(L=32))
    assert e.value.status == 1
    with pytest.raises(gf.GarfieldError) as e:
        plan.search_batched([[c.ncells]], gf.SearchParams(L=32))
    assert e.value.status == 1
    with pytest.raises(gf.GarfieldError) as e:
        plan.search(gf.SearchParams(L=32))  # graphs are not on the device
    assert e.value.status == 7
