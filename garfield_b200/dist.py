"""Multi-GPU host logic: one process per GPU.

The reference has no multi-GPU code.  Two ways to spread the query path over GPUs:

* replicas (indexes that fit one GPU, BASELINE configs 2 and 4): every rank holds the
  whole index and searches its own slice of the query batch (shard_range) with no
  data-path exchange; results are concatenated (gather_rows) only when one rank needs the
  full batch.
* cell sharding (indexes larger than one GPU): rank r holds the cells shard_cells(grid, G)[r]
  (gf_index_desc.shard_cells), every rank plans and searches the whole batch among its
  cells (gf_search_keys), and the per-query k best of all ranks are exchanged with one
  all-gather of qnum x k merge keys and merged (gf_merge_keys): sharded_search.
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


def shard_cells(grid, world: int) -> list[list[int]]:
    """Cells of each of `world` shards: the grid (row-major cell ids, last dimension
    fastest) is cut into `world` rectangular blocks by repeatedly halving the block with
    the most cells along its longest side, so the cells of a box query are mostly held by
    few ranks.  Shards are returned in a fixed order; every cell is in exactly one."""
    grid = [int(g) for g in grid]
    if world <= 0:
        raise ValueError("world must be > 0")
    ncells = int(np.prod(grid))
    if world > ncells:
        raise ValueError("more shards than cells")
    blocks = [[(0, g) for g in grid]]  # list of per-dimension [lo, hi)
    while len(blocks) < world:
        sizes = [int(np.prod([hi - lo for lo, hi in b])) for b in blocks]
        i = int(np.argmax(sizes))
        b = blocks.pop(i)
        d = max(range(len(b)), key=lambda j: (b[j][1] - b[j][0], -j))
        lo, hi = b[d]
        mid = (lo + hi) // 2
        left, right = list(b), list(b)
        left[d], right[d] = (lo, mid), (mid, hi)
        blocks[i:i] = [left, right]
    strides = np.cumprod([1] + grid[::-1][:-1])[::-1]
    out = []
    for b in blocks:
        axes = [np.arange(lo, hi) for lo, hi in b]
        mesh = np.meshgrid(*axes, indexing="ij")
        ids = sum(m.astype(np.int64) * int(s) for m, s in zip(mesh, strides))
        out.append(sorted(int(x) for x in np.ravel(ids)))
    return out


def merge_keys_host(keys: np.ndarray, k: int) -> np.ndarray:
    """CPU statement of the key merge (gf_merge_keys without the id lookup): keys
    (lists, qnum, k) uint64 -> (qnum, k) uint64, the k smallest non-empty keys per query."""
    keys = np.asarray(keys, dtype=np.uint64)
    lists, qnum, kk = keys.shape
    flat = np.sort(keys.transpose(1, 0, 2).reshape(qnum, lists * kk), axis=1)
    return flat[:, :k]


def exchange_keys(keys, group=None):
    """All-gather every rank's (qnum, k) merge keys into a (world, qnum, k) tensor (NCCL for
    CUDA tensors, any backend for host tensors).  The one collective of sharded search."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    keys = keys.contiguous()
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(keys.shape), dtype=keys.dtype, device=keys.device)
        dist.all_gather_into_tensor(out, keys, group=group)
        return out
    parts = [torch.empty_like(keys) for _ in range(world)]
    dist.all_gather(parts, keys, group=group)
    return torch.stack(parts, 0)


def sharded_search(index, plan, params, group=None, stream=None):
    """Cell-sharded search step on this rank: search the planned queries among the local
    shard's cells (gf_search_keys), all-gather the merge keys of every rank, merge them on
    this rank's GPU (gf_merge_keys).  Returns (ids int32, dists) CUDA tensors."""
    keys = plan.search_keys(params, stream)
    return index.merge_keys(exchange_keys(keys, group), params.k, stream)
