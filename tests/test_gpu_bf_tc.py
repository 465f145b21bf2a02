"""Tensor-core brute force (gf_bruteforce_ex path 2) against the CPU oracle's exact filtered
scan (naive_brute_force_with_filter restated, gpu_graph.cu:10782-10812): ids and canonical
distances must be identical, including ties (lower global id first), empty and tiny boxes,
padded row lengths and queries the tensor-core pass hands to the CUDA-core kernel."""
from __future__ import annotations

import numpy as np
import pytest

import garfield_b200 as gf
import oracle
from garfield_b200 import indexbuild, synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def bf_index(vectors, attrs, grid):
    """An index for the brute force only (a trivial one-edge graph per cell)."""
    lq, rq, _, cell_of = indexbuild.quantile_grid(attrs, grid)
    n = vectors.shape[0]
    return gf.Index.create(vectors=vectors, attrs=attrs.astype(np.float32), grid=np.asarray(grid, np.uint32),
                           l_quant=lq, r_quant=rq, cell_of=cell_of, graphs=np.zeros((n, 1), np.uint32), degree=1,
                           keep_fp32=True)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def run(g, q, lo, hi, k, **kw):
    stats = torch.zeros(3, dtype=torch.int32, device="cuda")
    ids, dist = g.bruteforce(dev(q), dev(lo), dev(hi), k, stats=stats, **kw)
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint32), dist.cpu().numpy(), stats.cpu().numpy()


def check(ds, g, k, path=2, max_fallback_frac=0.25, **kw):
    ids, dist, st = run(g, ds.queries, ds.lo, ds.hi, k, path=path, **kw)
    ref_ids, ref_d = oracle.bruteforce(ds.vectors, ds.attrs, ds.queries, ds.lo, ds.hi, k)
    bad = np.nonzero((ids != ref_ids).any(1) | (dist != ref_d).any(1))[0]
    assert bad.size == 0, f"{bad.size} queries differ, first {bad[:5]}"
    assert st[1] == 0, "a tensor-core wait ran out"
    # the tensor-core pass must prove most queries itself, not hand them all to CUDA cores
    assert st[0] <= max_fallback_frac * ds.queries.shape[0], st
    return st


@pytest.mark.parametrize("dim,grid,k", [(128, (4, 4), 10), (128, (4, 4), 1), (128, (4, 4), 16), (100, (2, 2, 2), 10),
                                        (256, (3, 2), 5), (16, (4,), 10), (384, (4, 4), 10), (1000, (2, 2), 7),
                                        (1024, (2, 2), 16)])
def test_tc_matches_oracle(dim, grid, k):
    ds = synth.make(30000, dim, 60, 700, grid, 0.1, seed=101 + dim + k, stratified=False)
    g = bf_index(ds.vectors, ds.attrs, grid)
    check(ds, g, k)
    g.close()


@pytest.mark.parametrize("dim,grid,k,max_fb", [(128, (4, 4), 17, 0.1), (128, (4, 4), 100, 0.1), (256, (2, 2), 50, 0.1),
                                               (1000, (2, 2), 64, 0.1), (64, (2, 2), 128, 1.0)])
def test_tc_deep_lists(dim, grid, k, max_fb):
    """k > 16: lists of 128 candidates, one epilogue warp per TMEM lane quarter; k = 128
    leaves no margin for the proof, so most queries go to the CUDA cores (still exact)."""
    ds = synth.make(30000, dim, 60, 700, grid, 0.1, seed=201 + dim + k, stratified=False)
    g = bf_index(ds.vectors, ds.attrs, grid)
    check(ds, g, k, max_fallback_frac=max_fb)
    g.close()


def test_tc_config3_shape_k100():
    """96-dim unit vectors, 3 attributes (uniform, Zipf, component band), k = 100."""
    ds = synth.config3(seed=33, n=60000, qnum=700, n_centers=60)
    g = bf_index(ds.vectors, ds.attrs, ds.grid)
    st = check(ds, g, 100, max_fallback_frac=0.05)
    assert st[2] > 0
    g.close()


def test_tc_wide_unit_norm_rows():
    """768-dim unit-normalised rows on an 8x8 grid (the shape of configuration 4): query
    chunks are streamed beside the point chunks instead of staying in shared memory."""
    ds = synth.config4(seed=43, n=30000, qnum=700, n_centers=40)
    g = bf_index(ds.vectors, ds.attrs, ds.grid)
    st = check(ds, g, 10, max_fallback_frac=0.05)
    assert st[2] > 0
    g.close()


def test_tc_fallback_hook_and_automatic_path():
    ds = synth.make(20000, 64, 40, 300, (2, 2), 0.15, seed=7, stratified=False)
    g = bf_index(ds.vectors, ds.attrs, (2, 2))
    st = check(ds, g, 10, test_fallback_every=3, max_fallback_frac=1.0)
    assert st[0] >= len([q for q in range(300) if q % 3 == 0])
    # the automatic path (k <= 128 with fp16 tiles) agrees with the CUDA-core path
    a_ids, a_d, _ = run(g, ds.queries, ds.lo, ds.hi, 10)
    c_ids, c_d, cst = run(g, ds.queries, ds.lo, ds.hi, 10, path=1)
    assert np.array_equal(a_ids, c_ids) and np.array_equal(a_d, c_d) and cst[0] == 0
    with pytest.raises(RuntimeError):
        g.bruteforce(dev(ds.queries), dev(ds.lo), dev(ds.hi), 129, path=2)  # past the deep lists
    g.close()


def test_tc_ties_duplicates_and_offset_data():
    rng = np.random.default_rng(5)
    base = (1.0e4 + rng.standard_normal((50, 96))).astype(np.float32)  # far from the origin: centring matters
    vectors = base[rng.integers(0, 50, 16000)]                        # many exact duplicates: ties by id
    attrs = rng.integers(0, 1000, (16000, 2)).astype(np.int32)
    queries = np.concatenate([vectors[:100], base[rng.integers(0, 50, 156)] + 0.25]).astype(np.float32)
    lo = rng.integers(0, 500, (256, 2)).astype(np.int32)
    hi = (lo + rng.integers(50, 500, (256, 2))).astype(np.int32)
    ds = synth.Dataset(vectors, attrs, queries, lo, hi, (4, 4))
    g = bf_index(vectors, attrs, (4, 4))
    # with 320 copies per distinct vector the 32 candidates often tie with the 33rd; those
    # queries are proven on the CUDA cores, and the result must be the oracle's either way
    check(ds, g, 10, max_fallback_frac=1.0)
    g.close()


def test_tc_edge_boxes_and_extreme_queries():
    ds = synth.make(12000, 128, 30, 130, (2, 2), 0.1, seed=9, stratified=False)
    lo, hi, q = ds.lo.copy(), ds.hi.copy(), ds.queries.copy()
    lo[0], hi[0] = [5000, 5000], [4000, 9000]        # empty box
    lo[1], hi[1] = [0, 0], [9999, 9999]              # every point
    lo[2], hi[2] = [123, 456], [125, 460]            # a handful of points (fewer than k)
    lo[3], hi[3] = [20000, 0], [30000, 9999]         # outside the attribute domain
    q[4] = 1.0e7                                     # beyond fp16 range once scaled: CUDA cores
    q[5] = q[5] * 0.0                                # the origin
    ds2 = synth.Dataset(ds.vectors, ds.attrs, q, lo, hi, (2, 2))
    g = bf_index(ds.vectors, ds.attrs, (2, 2))
    st = check(ds2, g, 10)
    assert st[0] >= 1                                # query 4 went to the CUDA cores
    # one query alone, and a batch that is not a multiple of the 128-query tile
    for sl in (slice(7, 8), slice(0, 129)):
        sub = synth.Dataset(ds.vectors, ds.attrs, q[sl], lo[sl], hi[sl], (2, 2))
        check(sub, g, 10, max_fallback_frac=1.0)
    g.close()


def test_tc_large_matches_cuda_cores():
    ds = synth.make(200_000, 128, 300, 2000, (4, 4), 0.1, seed=31)
    g = bf_index(ds.vectors, ds.attrs, (4, 4))
    t_ids, t_d, st = run(g, ds.queries, ds.lo, ds.hi, 10, path=2)
    c_ids, c_d, _ = run(g, ds.queries, ds.lo, ds.hi, 10, path=1)
    assert np.array_equal(t_ids, c_ids) and np.array_equal(t_d, c_d)
    assert st[1] == 0 and st[0] <= 200, st
    ref_ids, ref_d = oracle.bruteforce(ds.vectors, ds.attrs, ds.queries[:64], ds.lo[:64], ds.hi[:64], 10)
    assert np.array_equal(t_ids[:64], ref_ids) and np.array_equal(t_d[:64], ref_d)
    g.close()


def test_tc_calls_on_two_streams_share_the_working_memory():
    ds = synth.make(20000, 64, 40, 400, (2, 2), 0.1, seed=13, stratified=False)
    g = bf_index(ds.vectors, ds.attrs, (2, 2))
    q, lo, hi = dev(ds.queries), dev(ds.lo), dev(ds.hi)
    ref1 = g.bruteforce(q[:150].contiguous(), lo[:150].contiguous(), hi[:150].contiguous(), 10, path=2)
    ref2 = g.bruteforce(q[150:].contiguous(), lo[150:].contiguous(), hi[150:].contiguous(), 10, path=2)
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    a = (q[:150].contiguous(), lo[:150].contiguous(), hi[:150].contiguous())
    b = (q[150:].contiguous(), lo[150:].contiguous(), hi[150:].contiguous())
    torch.cuda.synchronize()
    with torch.cuda.stream(s1):
        r1 = g.bruteforce(*a, 10, stream=s1, path=2)
    with torch.cuda.stream(s2):
        r2 = g.bruteforce(*b, 10, stream=s2, path=2)
    torch.cuda.synchronize()
    for got, ref in ((r1, ref1), (r2, ref2)):
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    g.close()


def test_tc_wait_timeout_is_reported_and_answered_exactly():
    """Test hook: every tensor-core wait gives up after a few thousand polls and the query-tile
    loads never complete, so every CTA stops; the stops are counted and all queries are answered
    by the CUDA-core kernel, exactly.  The next call on the same context is normal."""
    ds = synth.make(20000, 64, 40, 300, (2, 2), 0.15, seed=17, stratified=False)
    g = bf_index(ds.vectors, ds.attrs, (2, 2))
    ref_ids, ref_d = oracle.bruteforce(ds.vectors, ds.attrs, ds.queries, ds.lo, ds.hi, 10)
    ids, dist, st = run(g, ds.queries, ds.lo, ds.hi, 10, path=2, test_wait=4096)
    assert st[1] > 0 and st[0] == ds.queries.shape[0], st
    assert np.array_equal(ids, ref_ids) and np.array_equal(dist, ref_d)
    ids, dist, st = run(g, ds.queries, ds.lo, ds.hi, 10, path=2)
    assert st[1] == 0 and st[0] <= ds.queries.shape[0] // 4, st
    assert np.array_equal(ids, ref_ids) and np.array_equal(dist, ref_d)
    g.close()
