"""Multi-GPU host logic: one process per GPU, each holding a replica of the index.

The reference has no multi-GPU code.  For indexes that fit one GPU (BASELINE configs
2 and 4) the query path shards by query: every rank searches its own slice of the batch
with no data-path exchange; results are concatenated (all_gather) only when one rank
needs the full batch.  The benchmark runs weak scaling instead (every rank searches a
full batch) and its only collective is the max over ranks of the timings.
"""
from __future__ import annotations

import numpy as np


def shard_range(qnum: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous slice [start, end) of a batch of qnum queries for `rank` of `world`;
    sizes differ by at most one and the slices tile the batch in rank order."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(qnum, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_rows(local: np.ndarray, qnum: int, world: int, group=None) -> np.ndarray:
    """All-gather per-rank row blocks (as produced by shard_range) into the full batch.
    Uses torch.distributed (gloo for host arrays, nccl for CUDA tensors upstream)."""
    import torch
    import torch.distributed as dist
    local = np.ascontiguousarray(local)
    t = torch.from_numpy(local.astype(np.int64) if local.dtype.kind in "ui" else local.astype(np.float64))
    width = t.shape[1] if t.ndim == 2 else 1
    rows = [shard_range(qnum, r, world) for r in range(world)]
    maxr = max(e - s for s, e in rows)
    pad = torch.zeros((maxr, width), dtype=t.dtype)
    pad[: t.shape[0]] = t.reshape(t.shape[0], width)
    bufs = [torch.zeros_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    out = torch.cat([b[: e - s] for b, (s, e) in zip(bufs, rows)], 0)
    return out.numpy().astype(local.dtype).reshape((qnum,) + tuple(local.shape[1:]))
