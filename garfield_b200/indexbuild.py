"""GMG index construction for synthetic datasets (test and benchmark inputs).

The reference builds its index offline with cuVS (indexbuild/*.py: CAGRA per-cell
graphs, CAGRA searches for cross-cell edges, k-means); cuVS is not available here, so
this module builds the same files with torch (GPU when present, else CPU):

  quantile_grid   indexbuild/tools.py:88-125 grid_scatter_V2 (per-dimension quantile slices)
  cell_graph      per-cell navigable graph of degree R (indexbuild/uniform_partition.py:516-563
                  uses CAGRA); here: half of each row from the exact 2R-NN, half from the 4R
                  nearest points of other k-means clusters (links to neighbouring clusters),
                  each robust-pruned with alpha = 1.2 (the DiskANN/Vamana rule)
  cross_edges     indexbuild/global_graph_build.py:116-157: for every point and every cell, the
                  E nearest points of that cell (local ids), here exact up to 2M points, and
                  above found by this library's own beam search of each cell's graph
                  (cross_edges_by_search), as the reference does with cagra.search
  kmeans          indexbuild/clustering.py:68-88 (cuVS k-means); here Lloyd iterations

Outputs use the reference's on-disk layout (global point order): graphs of all cells
concatenated in cell order with local ids, cross edges n x (cells * E) local ids.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _device(dev=None):
    if dev is not None:
        return torch.device(dev)
    return torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")


def quantile_grid(attrs: np.ndarray, grid):
    """Restates grid_scatter_V2 (indexbuild/tools.py:88-125): per dimension, a stable
    argsort cut into grid[j] runs of ceil(n / grid[j]) points (the last run takes the rest);
    l_quant / r_quant are the first / last sorted value of each run; cell id is the
    row-major mixed radix of the per-dimension slice ids (last dimension fastest)."""
    n, a = attrs.shape
    grid = np.asarray(grid, dtype=np.int64)
    lq, rq, slices = [], [], np.zeros((n, a), np.int32)
    for j in range(a):
        col = attrs[:, j]
        order = np.argsort(col, kind="stable")
        srt = col[order]
        g = int(grid[j])
        avg = (n + g - 1) // g
        starts = [s * avg for s in range(g)]
        ends = [min((s + 1) * avg, n) if s < g - 1 else n for s in range(g)]
        lq.append(np.array([srt[s] for s in starts], np.int32))
        rq.append(np.array([srt[e - 1] for e in ends], np.int32))
        for s in range(g):
            slices[order[starts[s]:ends[s]], j] = s
    factors = np.concatenate([np.cumprod(grid[::-1])[::-1][1:], [1]])
    cell_of = (slices.astype(np.int64) * factors[None, :]).sum(1).astype(np.uint32)
    return np.concatenate(lq), np.concatenate(rq), slices, cell_of


def _sqdist(x, y):
    """Squared L2 between row sets (torch, fp32)."""
    xx = (x * x).sum(1, keepdim=True)
    yy = (y * y).sum(1)[None, :]
    d = torch.addmm(xx + yy, x, y.t(), beta=1.0, alpha=-2.0)
    return d.clamp_min_(0.0)


def knn(x, k: int, chunk: int = 4096):
    """Exact k nearest neighbours of every row of x among the other rows of x."""
    n = x.shape[0]
    k = min(k, n - 1)
    idx = torch.empty((n, k), dtype=torch.int64, device=x.device)
    dst = torch.empty((n, k), dtype=torch.float32, device=x.device)
    ar = torch.arange(n, device=x.device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        d = _sqdist(x[s:e], x)
        d[torch.arange(e - s, device=x.device), ar[s:e]] = float("inf")
        v, i = torch.topk(d, k, dim=1, largest=False, sorted=True)
        idx[s:e], dst[s:e] = i, v
    return idx, dst


def _robust_prune(x, node_ids, cand, R: int, alpha: float, batch: int = 2048):
    """Robust pruning (Vamana RobustPrune) of candidate lists: walk the candidates of each
    node by increasing distance, keep c unless a kept p* has alpha * d(p*, c) <= d(node, c).
    cand: (m, M) int64 row ids (may contain -1 / duplicates).  Returns (m, R) ids, -1 padded."""
    m, M = cand.shape
    out = torch.full((m, R), -1, dtype=torch.int64, device=x.device)
    for s in range(0, m, batch):
        e = min(m, s + batch)
        c = cand[s:e]
        valid = c >= 0
        cs = torch.where(valid, c, torch.zeros_like(c))
        xv = x[cs]                                      # b x M x d
        xn = x[node_ids[s:e]]                           # b x d
        dnc = ((xv - xn[:, None, :]) ** 2).sum(-1)     # b x M
        dnc = torch.where(valid & (cs != node_ids[s:e, None]), dnc, torch.full_like(dnc, float("inf")))
        order = torch.argsort(dnc, dim=1, stable=True)
        c = torch.gather(cs, 1, order)
        dnc = torch.gather(dnc, 1, order)
        xv = x[c]
        # duplicates are adjacent after sorting by (distance, stable position)
        dup = torch.zeros_like(dnc, dtype=torch.bool)
        dup[:, 1:] = (c[:, 1:] == c[:, :-1])
        alive = torch.isfinite(dnc) & ~dup
        g = torch.bmm(xv, xv.transpose(1, 2))
        nrm = (xv * xv).sum(-1)
        dcc = (nrm[:, :, None] + nrm[:, None, :] - 2 * g).clamp_min_(0.0)
        cnt = torch.zeros(e - s, dtype=torch.int64, device=x.device)
        sel = torch.zeros_like(alive)
        for j in range(M):
            take = alive[:, j] & (cnt < R)
            sel[:, j] = take
            cnt += take.long()
            if j + 1 < M:
                kill = take[:, None] & (alpha * alpha * dcc[:, j, j + 1:] <= dnc[:, j + 1:])
                alive[:, j + 1:] &= ~kill
        # compact the selected ids, in distance order
        key = torch.where(sel, torch.arange(M, device=x.device)[None, :].expand_as(sel), torch.full_like(c, M))
        ks, ko = torch.sort(key, dim=1)
        picked = torch.gather(c, 1, ko)[:, :R]
        picked = torch.where(ks[:, :R] < M, picked, torch.full_like(picked, -1))
        out[s:e, : picked.shape[1]] = picked
    return out


def _first_distinct(cand, R: int):
    """Per row, the first R distinct non-negative ids of cand (in column order), -1 padded."""
    n, M = cand.shape
    big = torch.iinfo(torch.int64).max
    key = torch.where(cand >= 0, cand, torch.full_like(cand, big))
    srt, order = torch.sort(key, dim=1, stable=True)
    dup_s = torch.zeros_like(srt, dtype=torch.bool)
    dup_s[:, 1:] = srt[:, 1:] == srt[:, :-1]
    dup = torch.zeros_like(dup_s).scatter_(1, order, dup_s)
    keep = (cand >= 0) & ~dup
    rank = torch.cumsum(keep.long(), 1) - 1
    keep &= rank < R
    out = torch.full((n, R), -1, dtype=torch.int64, device=cand.device)
    rows = torch.arange(n, device=cand.device)[:, None].expand_as(cand)
    out[rows[keep], rank[keep]] = cand[keep]
    return out


def knn_other_label(x, labels, k: int, chunk: int = 4096):
    """k nearest neighbours of every row among the rows with a different label."""
    n = x.shape[0]
    idx = torch.full((n, k), -1, dtype=torch.int64, device=x.device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        d = _sqdist(x[s:e], x)
        d[labels[s:e, None] == labels[None, :]] = float("inf")
        kk = min(k, n)
        v, i = torch.topk(d, kk, dim=1, largest=False, sorted=True)
        idx[s:e, :kk] = torch.where(torch.isfinite(v), i, torch.full_like(i, -1))
    return idx


def cell_graph(x, R: int, labels=None, alpha: float = 1.2):
    """Degree-R navigable graph over the rows of x (local ids).

    Half of each row comes from the 2R nearest neighbours, robust-pruned.  The other half
    comes from the 4R nearest points whose cluster label differs from the node's, robust-
    pruned: links into the neighbouring clusters, so that greedy search can route between
    clusters instead of staying in the cluster of its entry point (with well separated
    clusters, nearest-neighbour edges never leave the cluster).  Rows are completed to R
    from the nearest-neighbour order.  Without labels the whole row is pruned 2R-NN."""
    n = x.shape[0]
    if n <= 1:
        return torch.zeros((n, R), dtype=torch.int64, device=x.device)
    nn_idx, _ = knn(x, 2 * R)
    ids = torch.arange(n, device=x.device)
    r_far = R // 2 if labels is not None else 0
    near = _robust_prune(x, ids, nn_idx, R - r_far, alpha)
    parts = [near]
    if r_far:
        far = _robust_prune(x, ids, knn_other_label(x, labels, 4 * R), r_far, alpha)
        parts.append(far)
    out = _first_distinct(torch.cat(parts + [nn_idx], 1), R)
    if bool((out < 0).any()):  # cells smaller than R + 1 points: repeat entries
        cnt = (out >= 0).sum(1, keepdim=True).clamp_min(1)
        col = torch.arange(R, device=x.device)[None, :] % cnt
        rep = torch.gather(torch.where(out >= 0, out, torch.zeros_like(out)), 1, col)
        out = torch.where(out >= 0, out, rep)
    return out


def cross_edges(x, cell_of_t, seg, E: int = 2, chunk: int = 8192):
    """For every point and every cell, the E nearest points of that cell (local ids)."""
    n = x.shape[0]
    P = len(seg) - 1
    out = torch.empty((n, P * E), dtype=torch.int64, device=x.device)
    for c in range(P):
        lo, hi = int(seg[c]), int(seg[c + 1])
        y = x[lo:hi]
        e = min(E, hi - lo)
        for s in range(0, n, chunk):
            t = min(n, s + chunk)
            d = _sqdist(x[s:t], y)
            _, i = torch.topk(d, e, dim=1, largest=False, sorted=True)
            if e < E:
                i = torch.cat([i, i[:, :1].expand(-1, E - e)], 1)
            out[s:t, c * E:(c + 1) * E] = i
    return out


def cross_edges_by_search(vectors: np.ndarray, attrs: np.ndarray, grid, l_quant, r_quant, cell_of: np.ndarray,
                          graphs: np.ndarray, R: int, E: int = 2, L: int = 32, width: int = 4,
                          chunk: int = 1 << 20, device=None) -> np.ndarray:
    """Cross-cell edges found by searching: for every point and every other cell, the E
    nearest points of that cell that a beam search of the cell's own graph finds (L, width),
    as local ids of that cell.  The reference builds its cross edges the same way, with
    cagra.search over each cell's index for all points (indexbuild/global_graph_build.py:
    116-157); the exact version (cross_edges) costs n^2 distances, which 10M points cannot
    afford.  The searches run on this library's own kernels: an index over the per-cell
    graphs without cross edges, every point as a query whose box is the target cell's
    slice box, searched inside that one cell (Plan.search_batched with the single batch
    [cell]).  A point's slots of its own cell hold its own local id (never read: a hop
    leaves a visited cell for an unvisited one).  Returns n x (cells * E) uint32."""
    import garfield_b200 as gf
    dev = _device(device)
    dev_index = dev.index if dev.type == "cuda" and dev.index is not None else 0
    n, a = attrs.shape
    grid = np.asarray(grid, np.int64)
    P = int(np.prod(grid))
    goff = np.concatenate([[0], np.cumsum(grid)[:-1]])
    lqf, rqf = np.asarray(l_quant, np.float32), np.asarray(r_quant, np.float32)
    sizes = np.bincount(cell_of, minlength=P)
    seg = np.concatenate([[0], np.cumsum(sizes)])
    order = np.argsort(cell_of, kind="stable")
    local = np.empty(n, np.uint32)
    local[order] = (np.arange(n) - seg[cell_of[order]]).astype(np.uint32)
    index = gf.Index.create(vectors=vectors, attrs=attrs.astype(np.float32), grid=grid.astype(np.uint32),
                            l_quant=l_quant, r_quant=r_quant, cell_of=cell_of, graphs=graphs, degree=R,
                            keep_fp32=False, device=dev_index)
    out = np.empty((n, P * E), np.uint32)
    xs = torch.from_numpy(np.ascontiguousarray(vectors, np.float32)).to(dev)
    plan = index.plan(min(chunk, n))
    params = gf.SearchParams(L=max(L, E), k=E, width=width)
    for c in range(P):
        rest, sl = c, np.zeros(a, np.int64)
        for j in range(a - 1, -1, -1):
            sl[j] = rest % grid[j]
            rest //= grid[j]
        lo = torch.from_numpy(np.array([lqf[goff[j] + sl[j]] for j in range(a)], np.float32)).to(dev)
        hi = torch.from_numpy(np.array([rqf[goff[j] + sl[j]] for j in range(a)], np.float32)).to(dev)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            lb = lo[None, :].expand(e - s, a).contiguous()
            rb = hi[None, :].expand(e - s, a).contiguous()
            plan.build(xs[s:e], lb, rb)
            ids, _ = plan.search_batched([[c]], params)
            g = ids.cpu().numpy().view(np.uint32)
            found = g != gf.NO_ID
            loc = np.where(found, local[np.minimum(g, n - 1)], 0).astype(np.uint32)
            # fewer than E found (a cell smaller than E): repeat the first
            loc = np.where(found, loc, loc[:, :1])
            out[s:e, c * E:(c + 1) * E] = loc
    own = cell_of.astype(np.int64)
    for j in range(E):
        out[np.arange(n), own * E + j] = local
    plan.close()
    index.close()
    del xs
    return out


def kmeans(x, C: int, iters: int = 10, seed: int = 0, chunk: int = 65536):
    """Lloyd k-means; returns int32 labels."""
    n = x.shape[0]
    g = torch.Generator(device="cpu").manual_seed(seed)
    cent = x[torch.randperm(n, generator=g)[:C].to(x.device)].clone()
    labels = torch.empty(n, dtype=torch.int64, device=x.device)
    for _ in range(iters):
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            labels[s:e] = _sqdist(x[s:e], cent).argmin(1)
        sums = torch.zeros_like(cent).index_add_(0, labels, x)
        cnt = torch.bincount(labels, minlength=C).float()
        nz = cnt > 0
        cent[nz] = sums[nz] / cnt[nz, None]
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        labels[s:e] = _sqdist(x[s:e], cent).argmin(1)
    return labels.to(torch.int32)


@dataclass
class GmgArrays:
    """Index arrays in the reference's layout (global point order)."""
    grid: np.ndarray        # uint32 a
    l_quant: np.ndarray     # int32 sum(grid)
    r_quant: np.ndarray
    slices: np.ndarray      # int32 n x a (per-dimension slice ids)
    cell_of: np.ndarray     # uint32 n
    graphs: np.ndarray      # uint32 n x R, per-cell graphs concatenated in cell order, local ids
    cross: np.ndarray       # uint32 n x (cells*E), local ids
    labels: np.ndarray      # int32 n
    degree: int
    cross_e: int


def build(vectors: np.ndarray, attrs: np.ndarray, grid, R: int = 32, E: int = 2, C: int = 1000,
          kmeans_iters: int = 10, seed: int = 0, device=None, cluster_links: bool = True,
          cross: str = "auto") -> GmgArrays:
    """The whole index.  cross: "exact" (every point against every cell, n^2 distances),
    "search" (cross_edges_by_search, needs a CUDA device and the built library) or "auto"
    (exact up to 2M points, search above)."""
    dev = _device(device)
    if cross == "auto":
        cross = "search" if vectors.shape[0] > 2_000_000 and dev.type == "cuda" else "exact"
    old_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        lq, rq, slices, cell_of = quantile_grid(attrs, grid)
        P = int(np.prod(grid))
        x = torch.from_numpy(np.ascontiguousarray(vectors, np.float32)).to(dev)
        n = x.shape[0]
        labels = kmeans(x, min(C, n), kmeans_iters, seed)
        order = np.argsort(cell_of, kind="stable")          # positions: cell-major, increasing id
        sizes = np.bincount(cell_of, minlength=P)
        seg = np.concatenate([[0], np.cumsum(sizes)])
        order_t = torch.from_numpy(order).to(dev)
        xo = x[order_t]
        lo_lab = labels[order_t]
        graphs = np.zeros((n, R), np.uint32)
        for c in range(P):
            lo, hi = int(seg[c]), int(seg[c + 1])
            if hi == lo:
                continue
            gcell = cell_graph(xo[lo:hi], R, labels=lo_lab[lo:hi] if cluster_links else None)
            graphs[lo:hi] = gcell.cpu().numpy().astype(np.uint32)
        labels = labels.cpu().numpy().astype(np.int32)
        if cross == "search":
            del xo
            cross_arr = cross_edges_by_search(vectors, attrs, grid, lq, rq, cell_of, graphs, R, E, device=dev)
        else:
            cr = cross_edges(xo, None, seg, E)
            cross_arr = np.empty((n, P * E), np.uint32)
            cross_arr[order] = cr.cpu().numpy().astype(np.uint32)
            del cr
        return GmgArrays(np.asarray(grid, np.uint32), lq, rq, slices, cell_of, graphs, cross_arr, labels, R, E)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old_tf32


def write_files(out_dir, name: str, ds, ix: GmgArrays, gt: np.ndarray | None = None) -> dict:
    """Write the reference's index/query files; returns the realdataset_search flags."""
    from . import write_attrs, write_fvecs, write_ranges, write_u32mat
    d = Path(out_dir)
    d.mkdir(parents=True, exist_ok=True)
    paths = dict(
        data_path=d / f"{name}_base.fvecs", query_path=d / f"{name}_query.fvecs", range=d / f"{name}.range",
        gt=d / f"{name}.gt", cagra_prefix=str(d / f"{name}_cell"), cagra_suffix=f".cagra{ix.degree}",
        global_graph=d / f"{name}_global.graph", grid=d / f"{name}.grid", attrs=d / f"{name}.attrs",
        cluster=d / f"{name}_cluster.bin",
    )
    write_fvecs(paths["data_path"], ds.vectors)
    write_fvecs(paths["query_path"], ds.queries)
    write_ranges(paths["range"], ds.lo, ds.hi)
    write_attrs(paths["attrs"], ds.attrs)
    P = int(np.prod(ix.grid))
    seg = np.concatenate([[0], np.cumsum(np.bincount(ix.cell_of, minlength=P))])
    for c in range(P):
        write_u32mat(f"{paths['cagra_prefix']}{c}{paths['cagra_suffix']}", ix.graphs[seg[c]:seg[c + 1]])
    write_u32mat(paths["global_graph"], ix.cross)
    # grid_info (indexbuild/tools.py:127-141)
    n, a = ix.slices.shape
    blob = [np.array([n, a], np.int32).tobytes(), ix.grid.astype(np.int32).tobytes()]
    off = 0
    for j in range(a):
        g = int(ix.grid[j])
        blob += [ix.l_quant[off:off + g].astype(np.int32).tobytes(), ix.r_quant[off:off + g].astype(np.int32).tobytes(),
                 ix.slices[:, j].astype(np.int32).tobytes()]
        off += g
    blob.append(ix.cell_of.astype(np.int32).tobytes())
    with open(paths["grid"], "wb") as f:
        f.write(b"".join(blob))
    with open(paths["cluster"], "wb") as f:
        f.write(np.array([n], np.int32).tobytes() + ix.labels.astype(np.int32).tobytes())
    if gt is not None:
        write_u32mat(paths["gt"], gt.astype(np.uint32))
    return {k: str(v) for k, v in paths.items()}
