"""Multi-rank host logic on CPU: 2 gloo ranks shard a query batch, search their slice
with the CPU oracle, and all-gather; the result equals the single-process search."""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

from garfield_b200.dist import shard_range

ROOT = Path(__file__).resolve().parents[1]


def test_shard_range_tiles_batch():
    for q in (0, 1, 7, 100, 10001):
        for w in (1, 2, 3, 8):
            spans = [shard_range(q, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == q
            assert all(spans[i][1] == spans[i + 1][0] for i in range(w - 1))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    import oracle
    from conftest import Case
    from garfield_b200.dist import gather_rows, shard_range
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    c = Case(6000, 32, 20, 101, (2, 2), 0.2, R=16, E=2, C=20, seed=9)
    s, e = shard_range(101, rank, world)
    ent = c.entry(16)
    # per-rank plan of its slice
    cnt, off, cells = oracle.plan_cells(c.ds.lo[s:e], c.ds.hi[s:e], c.ix.grid, c.ix.l_quant, c.ix.r_quant)
    cells, _ = oracle.order_cells(c.ds.queries[s:e], c.centroids, c.hist, cnt, off, cells)
    ids, _, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries[s:e], c.ds.lo[s:e], c.ds.hi[s:e], cnt,
                              off, cells, ent, L=32, K=10, threads=1)
    full = gather_rows(ids, 101, world)
    if rank == 0:
        ref, _, _ = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                                  c.cells, ent, L=32, K=10, threads=1)
        np.save(os.path.join(out_dir, "ok.npy"), np.array([np.array_equal(full, ref)]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_single_process(tmp_path):
    import torch.multiprocessing as mp
    port = 29500 + (os.getpid() % 1000)
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert bool(np.load(tmp_path / "ok.npy")[0])


def test_shard_cells_tile_grid():
    from garfield_b200.dist import shard_cells
    for grid in ((4, 4), (2, 2, 2), (16,), (3, 5)):
        n = int(np.prod(grid))
        for w in (1, 2, 3, 4, 8):
            if w > n:
                continue
            sh = shard_cells(grid, w)
            assert len(sh) == w and sorted(x for s in sh for x in s) == list(range(n))
            sizes = [len(s) for s in sh]
            if n % w == 0 and (n & (n - 1)) == 0:
                assert len(set(sizes)) == 1  # power-of-two grids split evenly
    # 4x4 over 4 ranks: the four 2x2 blocks
    assert shard_cells((4, 4), 4) == [[0, 1, 4, 5], [2, 3, 6, 7], [8, 9, 12, 13], [10, 11, 14, 15]]
    with pytest.raises(ValueError):
        shard_cells((2, 2), 5)


def _positions(cell_of):
    order = np.lexsort((np.arange(len(cell_of)), cell_of))
    pos = np.empty(len(cell_of), np.uint64)
    pos[order] = np.arange(len(cell_of), dtype=np.uint64)
    return pos


def _keys(ids, dist, pos_of):
    keys = np.full(ids.shape, np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64)
    ok = ids != 0xFFFFFFFF
    bits = dist.astype(np.float32).view(np.uint32).astype(np.uint64)
    keys[ok] = (bits[ok] << np.uint64(32)) | (pos_of[ids[ok]] << np.uint64(2))
    return keys


def _shard_worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    sys.path.insert(0, str(ROOT / "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    import oracle
    from conftest import Case
    from garfield_b200.dist import exchange_keys, merge_keys_host, shard_cells
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    c = Case(6000, 32, 20, 101, (2, 2), 0.2, R=16, E=2, C=20, seed=9)
    ent = c.entry(16)
    shards = shard_cells(c.ix.grid, world)
    args = (c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets, c.cells, ent)
    ids, d, _ = oracle.search(*args, L=32, K=10, threads=1, batches=[shards[rank]])
    pos_of = _positions(c.ix.cell_of)
    mine = torch.from_numpy(_keys(ids, d, pos_of).view(np.int64))
    allk = exchange_keys(mine).numpy().view(np.uint64)
    merged = merge_keys_host(allk, 10)
    if rank == 0:
        # the merge of the shards' results is the batched search with the shards as batches
        ref_ids, ref_d, _ = oracle.search(*args, L=32, K=10, threads=1, batches=shards)
        ok = np.array_equal(merged, _keys(ref_ids, ref_d, pos_of))
        np.save(os.path.join(out_dir, "ok.npy"), np.array([ok]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_cell_sharded(tmp_path):
    import torch.multiprocessing as mp
    port = 30500 + (os.getpid() % 1000)
    mp.spawn(_shard_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert bool(np.load(tmp_path / "ok.npy")[0])


def test_shard_result_depends_only_on_its_own_cell_order(small):
    """The premise of shard planning (a shard orders the cells of its multi-cell queries
    only): in the oracle's batched search with a shard as the batch, a query whose cells
    include fewer than two of the shard's gets the same answer whatever the order of its
    cells, so those queries may keep their cells in id order."""
    import oracle
    from garfield_b200.dist import shard_cells
    from conftest import mt_entry
    c = small
    ent = mt_entry(c.ix.degree, int(np.bincount(c.ix.cell_of, minlength=c.ncells).min()))
    for sh in shard_cells(c.ix.grid, 2):
        held = set(int(x) for x in sh)
        cells = c.cells.copy()
        changed = 0
        for q in range(c.counts.shape[0]):
            o, m = int(c.offsets[q]), int(c.counts[q])
            if sum(int(x) in held for x in cells[o:o + m]) < 2 and m > 1:
                cells[o:o + m] = np.sort(cells[o:o + m])
                changed += int(not np.array_equal(cells[o:o + m], c.cells[o:o + m]))
        kw = dict(L=32, K=10, batches=[sh])
        ref = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                            c.cells, ent, **kw)
        got = oracle.search(c.ix, c.ds.vectors, c.ds.attrs, c.ds.queries, c.ds.lo, c.ds.hi, c.counts, c.offsets,
                            cells, ent, **kw)
        assert np.array_equal(ref[0], got[0]) and np.array_equal(ref[1], got[1])
        assert changed > 0  # some queries really had their order dropped
