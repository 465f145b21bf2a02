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
