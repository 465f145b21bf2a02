#!/usr/bin/env python
"""Benchmark of the GMG query path: QPS at recall@10 >= 0.95 on BASELINE config 2
(1M x 128 fp32, 1000-center Gaussian mixture, 2 attributes on a 4x4 quantile grid,
R = 32 per-cell graphs + 2 cross-cell edges, 1000 k-means clusters, 10k queries with
10%-selectivity boxes, k = 10).

A step = planning (cell intersection + cluster-guided ordering) + the cell-by-cell search
of all 10k queries, with the index resident in HBM: the reference's QPS definition
qnum / (cost1 + cost2 + cost3) (realdataset_search.cu:2506-2508).  L is the smallest list
length in a fixed sweep whose recall on the ground-truth sample reaches the target.

  python bench.py [--gpus N --steps K --warmup W]           this implementation
  python bench.py --impl reference                          the reference's CPU exact filtered scan
                                                            (naive_brute_force_with_filter, built
                                                            from its sources) on the host cores
  python bench.py --mode out-of-core [--batch-cells B]     graphs in pinned host memory, streamed
                                                            per scheduled batch of B cells (row a17)
  torchrun ... bench.py --mode sharded                     cell-sharded index over the ranks, keys
                                                            all-gathered over NCCL and merged (row e)
  python bench.py --mode bruteforce                        exact filtered k-NN of all queries: tensor-core
                                                            pass vs the CUDA-core kernel
  python bench.py --impl reference-cuda                     the reference's own CUDA search
                                                            (oracle/_ref/realdataset_search) and our
                                                            CLI on the same reference-format files
  --config 3 / 4 (in-memory, bruteforce), --config 5 (out-of-core, sharded), --route 1
  (per-query choice of graph walk or tensor-core exact scan).
Multi-GPU (torchrun): every rank holds a replica of the index and searches its own batch
of queries from the same distribution (weak scaling, `value`); the one-GPU batch split over
the ranks is timed beside it (`strong`).  The collectives are the max-over-ranks of the
timings and the recall averages.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# data shape of each --config (config 3 runs at --n points)
SHAPES = {2: "1M x 128, 2 attrs, {sel:.0%} sel.",
          3: "config-3 shape: 96-dim unit-norm, 3 attrs (uniform, Zipf, component), {sel:.0%} sel.",
          4: "1M x 768 unit-norm, 2 attrs on 8x8, {sel:.0%} sel."}

# the reference's ef sweep (realdataset_search.cu:2757-2760), ascending, L >= k
L_SWEEP = [10, 15, 20, 25, 30, 35, 40, 45, 50, 55, 60, 70, 80, 90, 100, 120, 140, 160, 180, 200, 250, 300, 400,
           500, 600, 700, 800, 900, 1000, 1100, 1400, 1700]


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        def run():
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            while not self._stop.is_set():
                try:
                    out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                         timeout=5).stdout.strip()
                    if out:
                        self.samples.append([s.strip() for s in out.split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=6)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 3 + i and s[3 + i].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def ncu_traffic() -> tuple[float | None, str]:
    """DRAM bytes (read + write) of one search launch and where the figure comes from: the
    committed ncu summary of the search kernel (profiles/gmg_search_kernel_config2.md, line
    "traffic_bytes_per_launch: N", with the capture it was read from), not this run."""
    import re
    p = ROOT / "profiles" / "gmg_search_kernel_config2.md"
    if p.exists():
        txt = p.read_text()
        m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", txt)
        if m:
            cap = re.search(r"traffic_capture:\s*(.+)", txt)
            return float(m.group(1)), ("ncu capture recorded in profiles/gmg_search_kernel_config2.md"
                                       + (f" ({cap.group(1).strip()})" if cap else "") + ", not measured by this run")
    return None, "no ncu capture"


def peak_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


# --------------------------------------------------------------------------- data

def dataset_and_index(args, device):
    """Synthetic dataset of --config's shape and its index (cached per process tree under
    --cache).  Config 3 keeps its ratio of 1000 points per mixture component at any --n."""
    import torch
    from garfield_b200 import indexbuild, synth
    t0 = time.time()
    if args.config == 3:
        ds = synth.config3(seed=args.seed, n=args.n, qnum=args.qnum, n_centers=max(10, args.n // 1000),
                           selectivity=args.sel)
    elif args.config == 4:
        ds = synth.config4(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
    elif args.config == 5:
        # uint8 rows; one mixture component per 10k points, as 100k centres for 1B points
        ds, codes = synth.config5(seed=args.seed, n=args.n, qnum=args.qnum, n_centers=max(10, args.n // 10000),
                                  selectivity=args.sel)
        ds.codes = codes
    else:
        ds = synth.config2(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
    log(f"dataset {ds.vectors.shape} in {time.time() - t0:.1f}s")
    key = f"cfg{args.config}_n{args.n}_s{args.seed}_R{args.R}_E{args.E}_C{args.C}"
    cache = Path(args.cache) / key if args.cache else None
    names = ("grid", "l_quant", "r_quant", "slices", "cell_of", "graphs", "cross", "labels", "meta")
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if cache is not None and rank != 0 and world > 1:
        # rank 0 builds (or loads) the index; the others wait for its cache directory
        t0 = time.time()
        while not (cache / "meta.npy").exists():
            if time.time() - t0 > 3600:
                raise RuntimeError(f"no index cache at {cache} after an hour")
            time.sleep(2)
    if cache is not None and (cache / "meta.npy").exists():
        # arrays memory-mapped: the ranks of one box share the page cache
        z = {k: np.load(cache / f"{k}.npy", mmap_mode="r") for k in names}
        ix = indexbuild.GmgArrays(z["grid"], z["l_quant"], z["r_quant"], z["slices"], z["cell_of"], z["graphs"],
                                  z["cross"], z["labels"], int(z["meta"][0]), int(z["meta"][1]))
        log(f"index loaded from {cache}")
    else:
        t0 = time.time()
        ix = indexbuild.build(ds.vectors, ds.attrs, ds.grid, R=args.R, E=args.E, C=args.C, seed=args.seed,
                              device=device)
        torch.cuda.synchronize()
        log(f"index built in {time.time() - t0:.1f}s")
        if cache is not None:
            import shutil
            tmp = cache.with_name(f"{cache.name}.{os.getpid()}.tmp")
            try:
                tmp.mkdir(parents=True, exist_ok=True)
                arrs = {"grid": ix.grid, "l_quant": ix.l_quant, "r_quant": ix.r_quant, "slices": ix.slices,
                        "cell_of": ix.cell_of, "graphs": ix.graphs, "cross": ix.cross, "labels": ix.labels}
                for k, v in arrs.items():
                    np.save(tmp / f"{k}.npy", np.ascontiguousarray(v))
                np.save(tmp / "meta.npy", np.array([ix.degree, ix.cross_e], np.int64))  # written last
                if cache.exists():
                    shutil.rmtree(tmp, ignore_errors=True)
                else:
                    os.replace(tmp, cache)
            except OSError:
                shutil.rmtree(tmp, ignore_errors=True)
    return ds, ix


def cpu_baseline(ds, sample: int, threads: int, k: int = 10) -> dict:
    """The CPU exact filtered scan on host cores over `sample` queries: the reference's own
    naive_brute_force_with_filter (compiled from its sources, oracle/_ref/ref_golden) under
    omp parallel for when that binary is built (kind "reference"), with the oracle's
    restatement timed beside it; the restatement alone otherwise (kind "port")."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    q = ds.queries[:sample]
    oracle.bruteforce(ds.vectors, ds.attrs, q[:4], ds.lo[:4], ds.hi[:4], k, threads)  # warm
    t0 = time.perf_counter()
    oracle.bruteforce(ds.vectors, ds.attrs, q, ds.lo[:sample], ds.hi[:sample], k, threads)
    dt = time.perf_counter() - t0
    port = sample / dt
    binary = _ref_binary("ref_golden")
    if binary is None:
        return {"value": port, "unit": "queries/s", "cores": threads, "kind": "port",
                "sample": f"{sample} queries, exact filtered scan over all {ds.vectors.shape[0]} points "
                          f"({dt:.1f}s)"}
    sec = _time_reference_scan(binary, ds, np.arange(sample), sample, threads)[0]
    return {"value": sample / sec, "unit": "queries/s", "cores": threads, "kind": "reference",
            "sample": f"{sample} queries, exact filtered scan over all {ds.vectors.shape[0]} points ({sec:.1f}s): "
                      f"the reference's naive_brute_force_with_filter under omp parallel for",
            "port_value": round(port, 2)}


# --------------------------------------------------------------------------- arms

def run_ours(args):
    """Default mode.  One GPU: plan + search of config 2's 10k queries per step.  N GPUs
    (torchrun, one rank per GPU): every rank holds a replica of the index (config 2 fits
    one GPU) and searches its own batch of 10k queries per step, drawn from the same
    distribution (rank r: query stream r, synth.query_stream; rank 0's batch is the
    one-GPU batch), with no data-path collective: weak scaling, value = N x 10k queries /
    (max over ranks of the step time).  Beside it, "strong" times the one-GPU batch split
    over the ranks (dist.shard_range; total work fixed)."""
    import torch
    import torch.distributed as dist
    import garfield_b200 as gf
    from garfield_b200 import synth
    from garfield_b200.dist import shard_range

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)

    def reduce_max(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def reduce_sum(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    ds0, ix = dataset_and_index(args, device)
    ds = synth.query_stream(ds0, rank) if world > 1 else ds0
    t0 = time.time()
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                            r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree,
                            cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, f2h_factor=1.0, keep_fp32=True,
                            cross_spokesman=args.cross_spokesman, device=local)
    log(f"device index {index.device_bytes / 2**30:.2f} GiB in {time.time() - t0:.1f}s, "
        f"cross rows {index.cross_rows} of {index.n}")
    qnum = ds.queries.shape[0]
    qd = torch.from_numpy(ds.queries).to(device)
    lod = torch.from_numpy(ds.lo.astype(np.float32)).to(device)
    hid = torch.from_numpy(ds.hi.astype(np.float32)).to(device)
    # ground truth on a sample (exact, GPU brute force)
    S = min(args.gt_sample, qnum)
    t0 = time.time()
    K = args.k
    gt_ids, _ = index.bruteforce(qd[:S].contiguous(), lod[:S].contiguous(), hid[:S].contiguous(), K)
    gt = gt_ids.cpu().numpy().view(np.uint32)
    log(f"ground truth for {S} queries in {time.time() - t0:.1f}s")
    stream = torch.cuda.Stream(device)
    plan = index.plan(qnum)
    ids = torch.empty((qnum, K), dtype=torch.int32, device=device)
    dist_t = torch.empty((qnum, K), dtype=torch.float32, device=device)

    def sp(L, width):
        return gf.SearchParams(L=L, k=K, width=width, exact_tc=args.exact_tc, route=args.route)

    def step(L, width):
        plan.build(qd, lod, hid, args.prefilter, stream)
        plan.search(sp(L, width), stream, ids=ids, dist=dist_t)

    def find_L(width):
        """Smallest L of the sweep whose recall (mean over the ranks' samples) reaches the
        target at this width; every rank takes the same steps."""
        sweep = []
        for L in ([args.L] if args.L else [x for x in L_SWEEP if x >= K]):
            with torch.cuda.stream(stream):
                step(L, width)
            stream.synchronize()
            r = reduce_sum(gf.recall(ids[:S].cpu().numpy().view(np.uint32), gt)) / world
            sweep.append((L, round(r, 4)))
            log(f"width={width} L={L} recall@{K}={r:.4f}")
            if r >= args.target:
                return L, r, sweep
        return sweep[-1][0], sweep[-1][1], sweep

    def quick_ms(L, width, n=20):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                step(L, width)
            a.record(stream)
            for _ in range(n):
                step(L, width)
            b.record(stream)
        b.synchronize()
        return reduce_max(a.elapsed_time(b) / n)

    widths = [args.width] if args.width else [4, 8]  # widths 1 and 2 were slower at every L on B200
    best = None
    for wd in widths:
        L_w, r_w, sw = find_L(wd)
        if len(widths) == 1:
            ms = 0.0  # nothing to choose between
        else:
            ms = quick_ms(L_w, wd) if r_w >= args.target else float("inf")
        log(f"width={wd}: L={L_w} recall={r_w:.4f} {ms:.3f} ms/step")
        if best is None or ms < best[3]:
            best = (wd, L_w, r_w, ms, sw)
    args.width, L, recall, _, sweep = best
    # L2 flush buffer (> 126 MB L2)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)

    def timed(build, search, steps):
        """Device time of `steps` steps (build + search per step), L2 flushed between
        steps; returns (total ms max over ranks, plan ms list, search ms list, clocks)."""
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
               torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            for i in range(steps):
                with torch.cuda.stream(stream):
                    flush.fill_(float(i))
                    ev[i][0].record(stream)
                    build()
                    ev[i][1].record(stream)
                    search()
                    ev[i][2].record(stream)
            stream.synchronize()
        torch.cuda.synchronize()
        total = reduce_max(float(sum(a.elapsed_time(c) for a, b, c in ev)))
        return total, [a.elapsed_time(b) for a, b, c in ev], [b.elapsed_time(c) for a, b, c in ev], clocks

    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            step(L, args.width)
    total_ms, plan_ms, search_ms, clocks = timed(lambda: plan.build(qd, lod, hid, args.prefilter, stream),
                                                 lambda: plan.search(sp(L, args.width), stream, ids=ids, dist=dist_t),
                                                 args.steps)
    st = plan.stats()
    ms_per_step = total_ms / args.steps
    value = world * qnum / (ms_per_step / 1e3)
    # end to end through the C ABI from pinned host buffers
    qh = torch.from_numpy(ds.queries).pin_memory().numpy()
    lh = torch.from_numpy(ds.lo.astype(np.float32)).pin_memory().numpy()
    hh = torch.from_numpy(ds.hi.astype(np.float32)).pin_memory().numpy()
    e2e_plan = index.plan(qnum)
    params = sp(L, args.width)
    for _ in range(args.warmup):
        index.search_host(qh, lh, hh, e2e_plan, params, prefilter=args.prefilter, stream=stream)
    if world > 1:
        dist.barrier()
    e_ms = []
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(float(i))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        res_ids, _ = index.search_host(qh, lh, hh, e2e_plan, params, prefilter=args.prefilter, stream=stream)
        b.record(stream)
        b.synchronize()
        e_ms.append(a.elapsed_time(b))
    e2e_total = reduce_max(float(sum(e_ms)))
    e2e_value = world * qnum / (e2e_total / args.steps / 1e3)
    assert np.array_equal(res_ids, ids.cpu().numpy().view(np.uint32))
    strong = None
    if world > 1:
        # strong scaling: the one-GPU batch (query stream 0) split over the ranks
        s0, s1 = shard_range(ds0.queries.shape[0], rank, world)
        sq = torch.from_numpy(ds0.queries[s0:s1]).to(device)
        sl = torch.from_numpy(ds0.lo[s0:s1].astype(np.float32)).to(device)
        sh = torch.from_numpy(ds0.hi[s0:s1].astype(np.float32)).to(device)
        splan = index.plan(max(1, s1 - s0))
        sids = torch.empty((max(1, s1 - s0), K), dtype=torch.int32, device=device)
        sdist = torch.empty((max(1, s1 - s0), K), dtype=torch.float32, device=device)
        for _ in range(args.warmup):
            with torch.cuda.stream(stream):
                splan.build(sq, sl, sh, args.prefilter, stream)
                splan.search(sp(L, args.width), stream, ids=sids, dist=sdist)
        s_total, s_plan, s_search, _ = timed(lambda: splan.build(sq, sl, sh, args.prefilter, stream),
                                             lambda: splan.search(sp(L, args.width), stream, ids=sids, dist=sdist),
                                             args.steps)
        s_ms = s_total / args.steps
        strong = {"value": round(ds0.queries.shape[0] / (s_ms / 1e3), 1), "unit": "queries/s",
                  "ms_per_step": round(s_ms, 4), "queries_per_rank": s1 - s0,
                  "plan_ms": round(reduce_max(float(np.mean(s_plan))), 4),
                  "search_ms": round(reduce_max(float(np.mean(s_search))), 4),
                  "workload": f"the one-GPU batch of {ds0.queries.shape[0]} queries split over {world} ranks, same L"}
        splan.close()
    # roofline of the search kernel: algorithmic bytes from the device counters
    D, a_attr = ds.vectors.shape[1], ds.attrs.shape[1]
    bytes_step = (st["n_dist"] * (((D + 7) // 8 * 8) * 2 + a_attr * 4) + st["n_exp"] * ix.degree * 4 +
                  st["n_cross"] * (ix.cross_e * 4 + (4 if args.cross_spokesman else 0)))
    kern_s = float(np.mean(search_ms)) / 1e3
    achieved = bytes_step / kern_s / 1e9
    peak, peak_kind = peak_hbm()
    traffic, traffic_src = ncu_traffic()
    out = {
        "metric": f"QPS at recall@{K}>={args.target} ({SHAPES[args.config].format(sel=args.sel)})",
        "value": round(value, 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 accumulate",
        "data": f"synthetic (seeded Gaussian mixture; BASELINE config {args.config} shapes)",
        "config": {"workload": (f"config{args.config}: {ds.vectors.shape[0]} x {D} fp32, grid "
                                f"{'x'.join(str(int(g)) for g in ix.grid)}, R={ix.degree}, E={ix.cross_e}, C={args.C}, "
                                f"{qnum} queries per GPU, sel {args.sel:.0%}, k={K}"),
                   "L": L, "width": args.width, f"recall_at_{K}": round(recall, 4), "recall_sample": S,
                   "l2": "flushed (256 MiB write) between timed steps",
                   "parallelism": (f"replicas x{world}, a distinct batch of {qnum} queries per rank" if world > 1
                                   else "1 GPU"),
                   "plan_ms": round(float(np.mean(plan_ms)), 4), "search_ms": round(float(np.mean(search_ms)), 4),
                   "prefilter": args.prefilter, "exact_route": ("tensor-core exact scan" if args.exact_tc
                                                                else "fp16 warp scan"), "n_exact": int(st["n_exact"]),
                   "route": ("by cost: tensor-core exact scan when box count < 150 x cells x (L + 64)"
                             if args.route else "the reference's (postfilter / prefilter thresholds)"),
                   "sweep": sweep,
                   "cross_edges": (f"spokesman rows only: {index.cross_rows} of {index.n} (compress_global_graph_extreme)"
                                   if args.cross_spokesman else "full")},
        "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                "h2d_bytes_per_step": int(qh.nbytes + lh.nbytes + hh.nbytes), "d2h_bytes_per_step": int(qnum * K * 4)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                     "kernel": "gmg_search_kernel", "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": int(bytes_step),
                     "counters": {k: int(v) for k, v in st.items()}},
        "clocks": clocks.summary(),
        # per step: f2h, cell count, cell fill, centroid top-4, centroid merge, cell order, iota,
        # search (the CUB scan and radix-sort kernels of the planner are library launches)
        "gpu_launches": 8 * args.steps,
    }
    if args.exact_tc and st["n_exact"]:
        # the exact scan's time is inside search_ms, its work is not in the algorithmic bytes
        out["roofline"]["note"] = (f"{int(st['n_exact'])} of {int(st['n_queries'])} queries took the tensor-core "
                                   "exact scan (bf_tc_kernel): its time is inside search_ms but its bytes are not "
                                   "counted here; --mode bruteforce gives that kernel's roofline")
    if strong is not None:
        out["strong"] = strong
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(ds, args.cpu_sample, os.cpu_count() or 1, K)
    plan.close()
    e2e_plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_out_of_core(args):
    """Out-of-core mode (row a17): graphs and cross edges stay in pinned host memory; the
    scheduler groups the planned cells into batches of --batch-cells; each step plans the
    queries and runs the batched search, whose per-batch copies overlap the previous batch's
    search.  Reported beside the in-memory figure for the same batches (host_graph off)."""
    import torch
    import garfield_b200 as gf
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    ds, ix = dataset_and_index(args, device)
    common = dict(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                  r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree, cross=ix.cross,
                  cross_e=ix.cross_e, labels=ix.labels, f2h_factor=1.0, device=local)
    if args.config == 5:
        # uint8 rows decoded as code / 100 (the reference's u8 path), queries scaled by 0.01
        common.update(codec=2, codes=ds.codes, f2h_factor=0.01)
    streamed = gf.Index.create(**common, keep_fp32=True, host_graph=True, cross_spokesman=args.cross_spokesman)
    resident = gf.Index.create(**common, keep_fp32=False, host_graph=False, cross_spokesman=args.cross_spokesman)
    P = int(np.prod(ix.grid))
    seg = np.bincount(ix.cell_of, minlength=P)
    xrows = seg  # cross rows of each cell: its points, or its spokesmen
    if args.cross_spokesman:
        spk, _, _ = gf.spokesman(seg, ix.graphs)
        pos = np.arange(len(spk))
        xrows = np.bincount(np.repeat(np.arange(P), seg)[spk == pos], minlength=P)
    qnum = ds.queries.shape[0]
    qd = torch.from_numpy(ds.queries).to(device)
    lod = torch.from_numpy(ds.lo.astype(np.float32)).to(device)
    hid = torch.from_numpy(ds.hi.astype(np.float32)).to(device)
    S = min(args.gt_sample, qnum)
    gt = streamed.bruteforce(qd[:S].contiguous(), lod[:S].contiguous(), hid[:S].contiguous(), 10)[0]
    gt = gt.cpu().numpy().view(np.uint32)
    stream = torch.cuda.Stream(device)
    width = args.width or 4
    ids = torch.empty((qnum, 10), dtype=torch.int32, device=device)
    dist_t = torch.empty((qnum, 10), dtype=torch.float32, device=device)
    res = {}
    for name, index in (("streamed", streamed), ("resident", resident)):
        plan = index.plan(qnum)
        plan.build(qd, lod, hid, 0.0, stream)
        t0 = time.perf_counter()
        batches, splits = plan.schedule(args.batch_cells)
        sched_ms = (time.perf_counter() - t0) * 1e3

        def step(L):
            plan.build(qd, lod, hid, 0.0, stream)
            plan.search_batched(batches, gf.SearchParams(L=L, k=10, width=width), stream, ids=ids, dist=dist_t)

        L, recall, sweep = None, 0.0, []
        for Lc in ([args.L] if args.L else L_SWEEP):
            with torch.cuda.stream(stream):
                step(Lc)
            stream.synchronize()
            recall = gf.recall(ids[:S].cpu().numpy().view(np.uint32), gt)
            sweep.append((Lc, round(recall, 4)))
            L = Lc
            if recall >= args.target:
                break
        flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
        for _ in range(args.warmup):
            with torch.cuda.stream(stream):
                step(L)
        stream.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ms = []
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(float(i))
                a.record(stream)
                step(L)
                b.record(stream)
            b.synchronize()
            ms.append(a.elapsed_time(b))
        h2d = sum(int(seg[c]) * ix.degree * 4 + len(bt) * int(xrows[c]) * ix.cross_e * 4 for bt in batches for c in bt)
        res[name] = {"qps": round(qnum / (float(np.mean(ms)) / 1e3), 1), "ms_per_step": round(float(np.mean(ms)), 4),
                     "L": L, "recall_at_10": round(recall, 4), "sweep": sweep,
                     "h2d_graph_bytes_per_step": h2d if name == "streamed" else 0}
        res["batches"], res["splits"], res["schedule_ms"] = batches, splits, round(sched_ms, 3)
        plan.close()
    shape = (f"{ds.vectors.shape[0] / 1e6:g}M x 128 uint8, 2 attrs on 16x16, {args.sel:.0%} sel." if args.config == 5
             else "1M x 128, 2 attrs, 10% sel.")
    out = {"metric": f"QPS at recall@10>=0.95, graphs streamed per batch of cells ({shape})",
           "value": res["streamed"]["qps"], "unit": "queries/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": res["streamed"]["ms_per_step"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None,
           "dtype": "u8 storage, f32 accumulate" if args.config == 5 else "f16 storage, f32 accumulate",
           "data": f"synthetic (seeded Gaussian mixture; BASELINE config {args.config} shapes)",
           "config": {"workload": f"config{args.config}: {ds.vectors.shape[0]} points, {qnum} queries, out-of-core batches",
                      "batch_cells": args.batch_cells, "width": width,
                      "n_batches": len(res["batches"]), "splits": res["splits"], "schedule_ms": res["schedule_ms"],
                      "batches": res["batches"], "streamed": res["streamed"], "resident_same_batches": res["resident"],
                      "cross_edges": (f"spokesman rows only: {streamed.cross_rows} of {streamed.n}"
                                      if args.cross_spokesman else "full"),
                      "l2": "flushed (256 MiB write) between timed steps"}}
    print(json.dumps(out), flush=True)


def peak_tensor() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured (cuBLAS bf16 burst; fp16 runs at the same rate)"
        except Exception:
            pass
    return 1590.0, "fallback"


def run_bruteforce(args):
    """Exact filtered k-NN mode (gf_bruteforce, the GPU ground truth): --config's data, all
    queries, k = 10 (100 for config 3).  Times the tensor-core pass (query x point products on
    tcgen05 with a proven error bound, exact re-rank, CUDA-core answer for unproven queries)
    and, while points x queries stays below 1e10, the CUDA-core kernel on the same inputs,
    checking that both return the same ids and distances.  The roofline is the tensor pipe:
    executed MMA FLOPs per second.  Under torchrun every rank holds the index and takes its
    slice of the query batch (dist.shard_range; strong scaling, the batch is fixed)."""
    import torch
    import torch.distributed as dist
    import garfield_b200 as gf
    from garfield_b200 import indexbuild, synth
    from garfield_b200.dist import shard_range
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)

    def reduce_max(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    K = args.k
    if args.config == 3:
        ds = synth.config3(seed=args.seed, n=args.n, qnum=args.qnum, n_centers=max(10, args.n // 1000),
                           selectivity=args.sel)
        shape = f"{args.n / 1e6:g}M x 96 unit-norm, 3 attrs on 4x4x4, {args.sel:.0%} sel., k=100"
    elif args.config == 4:
        ds = synth.config4(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
        shape = f"{args.n / 1e6:g}M x 768 unit-norm, 2 attrs on 8x8, {args.sel:.0%} sel., k=10"
    else:
        ds = synth.config2(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
        shape = f"{args.n / 1e6:g}M x 128, 2 attrs, {args.sel:.0%} sel., k=10"
    lq, rq, _, cell_of = indexbuild.quantile_grid(ds.attrs, ds.grid)
    n, D = ds.vectors.shape
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=np.asarray(ds.grid, np.uint32),
                            l_quant=lq, r_quant=rq, cell_of=cell_of, graphs=np.zeros((n, 1), np.uint32), degree=1,
                            keep_fp32=True, device=local)
    qtot = ds.queries.shape[0]
    s0, s1 = shard_range(qtot, rank, world) if world > 1 else (0, qtot)
    qnum = s1 - s0
    qd = torch.from_numpy(ds.queries[s0:s1]).to(device)
    lod = torch.from_numpy(ds.lo[s0:s1].astype(np.float32)).to(device)
    hid = torch.from_numpy(ds.hi[s0:s1].astype(np.float32)).to(device)
    stream = torch.cuda.Stream(device)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
    stats = torch.zeros(3, dtype=torch.int32, device=device)

    def timed(path, steps, warmup):
        for _ in range(warmup):
            index.bruteforce(qd, lod, hid, K, stream=stream, path=path, stats=stats)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        ms = []
        with ClockSampler(local) as clocks:
            for i in range(steps):
                with torch.cuda.stream(stream):
                    flush.fill_(float(i))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                ids, dist_t = index.bruteforce(qd, lod, hid, K, stream=stream, path=path, stats=stats)
                b.record(stream)
                b.synchronize()
                ms.append(a.elapsed_time(b))
        return ids, dist_t, float(np.mean(ms)), stats.cpu().numpy().copy(), clocks.summary()

    t_ids, t_d, t_ms, st, clocks = timed(2, args.steps, args.warmup)
    total_ms = reduce_max(t_ms * args.steps)
    ms_step = total_ms / args.steps
    cuda_core = float(n) * float(qtot) < 1e10  # the CUDA-core kernel scans every point per query
    if cuda_core:
        c_ids, c_d, c_ms, _, _ = timed(1, 1, 1)
        same = bool(torch.equal(t_ids, c_ids) and torch.equal(t_d, c_d))
    # end to end: host queries and boxes in pinned memory, ids back to the host
    qh, lh, hh = (torch.from_numpy(np.ascontiguousarray(x)).pin_memory()
                  for x in (ds.queries[s0:s1], ds.lo[s0:s1].astype(np.float32), ds.hi[s0:s1].astype(np.float32)))
    qg, lg, hg = torch.empty_like(qd), torch.empty_like(lod), torch.empty_like(hid)
    ih = torch.empty((qnum, K), dtype=torch.int32).pin_memory()
    e_ms = []
    if world > 1:
        dist.barrier()
    for i in range(max(args.warmup, 1) + args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(float(i))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            qg.copy_(qh, non_blocking=True)
            lg.copy_(lh, non_blocking=True)
            hg.copy_(hh, non_blocking=True)
            ids, _ = index.bruteforce(qg, lg, hg, K, stream=stream)
            ih.copy_(ids, non_blocking=True)
            b.record(stream)
        b.synchronize()
        if i >= max(args.warmup, 1):
            e_ms.append(a.elapsed_time(b))
    assert torch.equal(ih, t_ids.cpu())
    e2e_ms = reduce_max(float(np.sum(e_ms))) / args.steps
    products = int(st[2])
    dp = (D + 15) // 16 * 16
    flops = 2.0 * products * 128 * 128 * dp
    achieved = flops / (t_ms / 1e3) / 1e12
    peak, peak_kind = peak_tensor()
    out = {"metric": f"exact filtered k-NN queries/s ({shape})",
           "value": round(qtot / (ms_step / 1e3), 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
           "scaling": "strong" if world > 1 else "weak",
           "vs_baseline": None, "dtype": "f16 products, f32 accumulate, f32 exact re-rank",
           "data": f"synthetic (seeded Gaussian mixture; BASELINE config {args.config} shapes)",
           "config": {"workload": f"config{args.config} brute force: {n} x {D} fp32, {qtot} queries"
                                  f"{f' split over {world} ranks' if world > 1 else ''}, sel {args.sel:.0%}, k={K}",
                      "recall": "1.0 (exact)", "l2": "flushed (256 MiB write) between timed steps",
                      "fallback_queries_rank0": int(st[0]), "timeouts_rank0": int(st[1]),
                      "tile_products_rank0": products,
                      "dense_products_rank0": ((qnum + 127) // 128) * ((n + 127) // 128)},
           "e2e": {"value": round(qtot / (e2e_ms / 1e3), 1), "unit": "queries/s",
                   "h2d_bytes_per_step": int(qh.nbytes + lh.nbytes + hh.nbytes) * world,
                   "d2h_bytes_per_step": int(ih.nbytes) * world},
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(achieved / peak, 4), "traffic": None,
                        "kernel": "bf_tc_kernel (whole call timed, rank 0)",
                        "peak_kind": peak_kind, "flops_per_step_rank0": flops},
           "clocks": clocks,
           # morton, 3 radix-sort passes are CUB's; prep, boxes, tiles, tc, merge, CUDA-core list
           "gpu_launches": 6 * args.steps}
    if cuda_core:
        out["config"].update({"cuda_core_ms_per_step": round(c_ms, 3), "speedup_vs_cuda_cores": round(c_ms / t_ms, 2),
                              "identical_to_cuda_cores": same})
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(ds, args.cpu_sample, os.cpu_count() or 1, K)
    index.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_fullgraph(args):
    """Full-graph post-filter ablation (row f4): the reference's baseline that searches
    assemble_edges' graph of the whole index and applies the box only at the end
    (full_graph_search.cuh:179-997), on config 2 beside the cell-by-cell search: recall at
    each L of the sweep and QPS (plan + search) for both."""
    import torch
    import garfield_b200 as gf
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    ds, ix = dataset_and_index(args, device)
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                            r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree,
                            cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, f2h_factor=1.0, keep_fp32=True,
                            device=local)
    index.assemble(ix.cross_e)
    qnum = ds.queries.shape[0]
    qd = torch.from_numpy(ds.queries).to(device)
    lod = torch.from_numpy(ds.lo.astype(np.float32)).to(device)
    hid = torch.from_numpy(ds.hi.astype(np.float32)).to(device)
    S = min(args.gt_sample, qnum)
    gt = index.bruteforce(qd[:S].contiguous(), lod[:S].contiguous(), hid[:S].contiguous(), 10)[0]
    gt = gt.cpu().numpy().view(np.uint32)
    stream = torch.cuda.Stream(device)
    plan = index.plan(qnum)
    width = args.width or 4
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
    res = {}
    for name in ("cell_by_cell", "full_graph_postfilter"):
        def step(L):
            plan.build(qd, lod, hid, 0.0, stream)
            p = gf.SearchParams(L=L, k=10, width=width)
            return plan.search(p, stream) if name == "cell_by_cell" else plan.search_fullgraph(p, stream)
        sweep = []
        for L in L_SWEEP[:12]:
            with torch.cuda.stream(stream):
                ids, _ = step(L)
            stream.synchronize()
            sweep.append((L, round(gf.recall(ids[:S].cpu().numpy().view(np.uint32), gt), 4)))
        L40 = 40
        for _ in range(args.warmup):
            with torch.cuda.stream(stream):
                step(L40)
        ms = []
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(float(i))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                step(L40)
                b.record(stream)
            b.synchronize()
            ms.append(a.elapsed_time(b))
        res[name] = {"qps_at_L40": round(qnum / (float(np.mean(ms)) / 1e3), 1),
                     "ms_per_step_at_L40": round(float(np.mean(ms)), 4), "sweep": sweep}
    out = {"metric": "recall@10 and QPS of the full-graph post-filter ablation vs the cell-by-cell search (1M x 128)",
           "value": res["full_graph_postfilter"]["qps_at_L40"], "unit": "queries/s", "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["full_graph_postfilter"]["ms_per_step_at_L40"],
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 accumulate",
           "data": "synthetic (seeded Gaussian mixture; BASELINE config 2 shapes)",
           "config": {"workload": "config2, full-graph ablation (assemble_edges, reserve = E)", "width": width,
                      "recall_sample": S, "l2": "flushed (256 MiB write) between timed steps", **res}}
    print(json.dumps(out), flush=True)


def run_sharded(args):
    """Cell-sharded mode (row e, strong scaling): rank r of N holds the cells
    dist.shard_cells(grid, N)[r] only; a step plans the queries on every rank (cell lists of
    all of them, centroid order only for those with two or more local cells), searches them
    among the local cells (gf_search_keys), all-gathers the (qnum, k) merge keys over NCCL
    and merges them (gf_merge_keys) on every rank."""
    import torch
    import torch.distributed as dist
    import garfield_b200 as gf
    from garfield_b200.dist import exchange_keys, shard_cells
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    ds, ix = dataset_and_index(args, device)
    mine = shard_cells(ix.grid, world)[rank]
    codec = dict(codec=2, codes=ds.codes, f2h_factor=0.01) if args.config == 5 else dict(f2h_factor=1.0)
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                            r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree,
                            cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, keep_fp32=False,
                            shard_cells=mine if world > 1 else None, device=local, **codec)
    qnum = ds.queries.shape[0]
    qd = torch.from_numpy(ds.queries).to(device)
    lod = torch.from_numpy(ds.lo.astype(np.float32)).to(device)
    hid = torch.from_numpy(ds.hi.astype(np.float32)).to(device)
    S = min(args.gt_sample, qnum)
    stream = torch.cuda.Stream(device)
    plan = index.plan(qnum)
    width = args.width or 4
    keys = torch.empty((qnum, 10), dtype=torch.int64, device=device)

    def step(L):
        plan.build(qd, lod, hid, 0.0, stream)
        plan.search_keys(gf.SearchParams(L=L, k=10, width=width), stream, keys=keys)
        with torch.cuda.stream(stream):
            allk = exchange_keys(keys) if world > 1 else keys[None]
        return index.merge_keys(allk, 10, stream)

    # ground truth: exact scan on a whole index on rank 0, broadcast
    gt = torch.zeros((S, 10), dtype=torch.int32, device=device)
    if rank == 0:
        whole = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid,
                                l_quant=ix.l_quant, r_quant=ix.r_quant, cell_of=ix.cell_of,
                                graphs=np.zeros((ds.vectors.shape[0], 1), np.uint32), degree=1, keep_fp32=True,
                                device=local)
        gt.copy_(whole.bruteforce(qd[:S].contiguous(), lod[:S].contiguous(), hid[:S].contiguous(), 10)[0])
        whole.close()
        del whole
    if world > 1:
        dist.broadcast(gt, 0)
    gt_np = gt.cpu().numpy().view(np.uint32)
    L, recall, sweep = None, 0.0, []
    for Lc in ([args.L] if args.L else L_SWEEP):
        ids, _ = step(Lc)
        stream.synchronize()
        recall = gf.recall(ids[:S].cpu().numpy().view(np.uint32), gt_np)
        sweep.append((Lc, round(recall, 4)))
        L = Lc
        if recall >= args.target:
            break
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
    for _ in range(args.warmup):
        step(L)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(float(i))
                ev[i][0].record(stream)
            step(L)
            with torch.cuda.stream(stream):
                ev[i][1].record(stream)
        stream.synchronize()
    total_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    if world > 1:
        t = torch.tensor([total_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms = total_ms / args.steps
    shape = (f"{ds.vectors.shape[0] / 1e6:g}M x 128 uint8, 2 attrs on 16x16, {args.sel:.0%} sel." if args.config == 5
             else "1M x 128, 2 attrs, 10% sel.")
    out = {"metric": f"QPS at recall@10>=0.95, cell-sharded index ({shape})",
           "value": round(qnum / (ms / 1e3), 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None,
           "dtype": "u8 storage, f32 accumulate" if args.config == 5 else "f16 storage, f32 accumulate",
           "data": f"synthetic (seeded Gaussian mixture; BASELINE config {args.config} shapes)",
           "config": {"workload": f"config{args.config}: {ds.vectors.shape[0]} points, {qnum} queries, cell-sharded",
                      "parallelism": f"cell shards x{world}", "L": L,
                      "width": width, "recall_at_10": round(recall, 4), "recall_sample": S, "sweep": sweep,
                      "shard_cells": mine, "device_bytes_rank0": index.device_bytes,
                      "exchange_bytes_per_rank": qnum * 10 * 8,
                      "l2": "flushed (256 MiB write) between timed steps"},
           "clocks": clocks.summary()}
    plan.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def _ref_binary(name: str) -> Path | None:
    p = ROOT / "oracle" / "_ref" / name
    return p if p.exists() and os.access(p, os.X_OK) else None


def _write_query_files(d: Path, ds) -> dict:
    from garfield_b200 import write_attrs, write_fvecs, write_ranges
    d.mkdir(parents=True, exist_ok=True)
    paths = {"data": d / "base.fvecs", "attrs": d / "base.attrs", "queries": d / "query.fvecs",
             "ranges": d / "query.range"}
    write_fvecs(paths["data"], ds.vectors)
    write_attrs(paths["attrs"], ds.attrs)
    write_fvecs(paths["queries"], ds.queries)
    write_ranges(paths["ranges"], ds.lo, ds.hi)
    return {k: str(v) for k, v in paths.items()}


def _time_reference_scan(binary: Path, ds, rows: np.ndarray, chunk: int, threads: int) -> list:
    """Wall seconds of the reference's naive_brute_force_with_filter (oracle/_ref/ref_golden
    bf_omp) over consecutive chunks of the query rows `rows`, `threads` OpenMP threads."""
    import shutil
    import tempfile
    from garfield_b200 import write_fvecs, write_ranges
    tmp = Path(tempfile.mkdtemp(prefix="gf_refcpu_"))
    try:
        base = _write_query_files(tmp, ds)
        write_fvecs(tmp / "q.fvecs", ds.queries[rows])
        write_ranges(tmp / "q.range", ds.lo[rows], ds.hi[rows])
        r = subprocess.run([str(binary), "bf_omp", base["data"], base["attrs"], str(tmp / "q.fvecs"),
                            str(tmp / "q.range"), "10", str(threads), str(chunk), str(tmp / "out.u32")],
                           capture_output=True, text=True, timeout=1200)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    if r.returncode != 0:
        raise RuntimeError(f"ref_golden bf_omp failed: {r.stderr[-500:]}")
    return [float(line.split()[1]) for line in r.stdout.splitlines() if line.startswith("seconds ")]


def run_reference_cpu(args):
    """Reference arm: the reference's own CPU exact filtered scan on the host cores.

    naive_brute_force_with_filter (gpu_graph.cu:10782-10812) compiled from the reference's
    sources (oracle/_ref/ref_golden, mode bf_omp) and called per query under omp parallel
    for, as realdataset_search.cu:2330-2335 does, with all host threads; each step is a
    bounded sample of the 10k queries.  Without that binary the oracle's restatement of
    the same scan (oracle/gf_oracle.c) is timed instead (kind "port")."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    from garfield_b200 import synth
    ds = synth.config2(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
    threads = os.cpu_count() or 1
    S = args.ref_sample
    binary = _ref_binary("ref_golden")
    kind = "reference" if binary else "port"
    steps = args.warmup + args.steps
    starts = [(i * S) % max(1, ds.queries.shape[0] - S) for i in range(steps)]
    rows = np.concatenate([np.arange(s0, s0 + S) for s0 in starts])
    if binary:
        times = _time_reference_scan(binary, ds, rows, S, threads)[args.warmup:]
    else:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle
        times = []
        for i, s0 in enumerate(starts):
            sl = slice(s0, s0 + S)
            t0 = time.perf_counter()
            oracle.bruteforce(ds.vectors, ds.attrs, ds.queries[sl], ds.lo[sl], ds.hi[sl], 10, threads)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
    value = S / float(np.mean(times))
    what = ("naive_brute_force_with_filter compiled from the reference's sources, one call per query under "
            "omp parallel for" if binary else "the oracle's restatement of naive_brute_force_with_filter")
    out = {
        "impl": "reference", "metric": "QPS at recall@10>=0.95 (1M x 128, 2 attrs, 10% sel.)",
        "value": round(value, 2), "unit": "queries/s", "n_gpus": int(os.environ.get("WORLD_SIZE", 1)),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(float(np.mean(times)) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture; BASELINE config 2 shapes)",
        "config": {"workload": (f"config2: {ds.vectors.shape[0]} x 128 fp32, 2 attrs, {ds.queries.shape[0]} queries, "
                                f"sel {args.sel:.0%}, k=10"),
                   "step": f"{S} queries (bounded sample), exact scan (recall 1.0): {what}"},
        "cpu_baseline": {"value": round(value, 2), "unit": "queries/s", "cores": threads, "kind": kind,
                         "sample": f"{S} queries per step, exact filtered scan over {ds.vectors.shape[0]} points "
                                   f"({what}; file loading not timed)"},
        "e2e": {"value": round(value, 2), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def _cell_major(ds, ix, gt):
    """The same dataset and index with point ids renumbered cell-major (ids of cell 0
    first, increasing old id inside a cell).  The reference's load_clustering histograms
    cells as id / 62500 (tools.cuh:590), which is only the grid's cell when ids are
    cell-major; positions, graphs (local ids) and cross edges (local ids) are unchanged
    by the renumbering, so both arms search the same index."""
    from types import SimpleNamespace
    from garfield_b200 import indexbuild
    order = np.argsort(ix.cell_of, kind="stable")
    inv = np.empty_like(order)
    inv[order] = np.arange(order.size)
    ds2 = SimpleNamespace(vectors=ds.vectors[order], attrs=ds.attrs[order], queries=ds.queries, lo=ds.lo, hi=ds.hi)
    ix2 = indexbuild.GmgArrays(ix.grid, ix.l_quant, ix.r_quant, ix.slices[order], ix.cell_of[order], ix.graphs,
                               ix.cross[order], ix.labels[order], ix.degree, ix.cross_e)
    gt2 = np.where(gt == 0xFFFFFFFF, gt, inv[np.minimum(gt, order.size - 1)]).astype(np.uint32)
    return ds2, ix2, gt2


def _read_csv(path: Path) -> list:
    rows = []
    for line in path.read_text().strip().splitlines()[1:]:
        f = line.split(",")
        rows.append({"ef": int(f[0]), "recall": float(f[1]), "qps": float(f[2]), "cost1": float(f[4]),
                     "cost2": float(f[5]), "cost3": float(f[6])})
    return rows


def _best(rows: list, target: float):
    ok = [r for r in rows if r["recall"] >= target]
    return max(ok, key=lambda r: r["qps"]) if ok else None


def run_reference_cuda(args):
    """The reference's own CUDA search beside ours on the same files (row N4 of the plan).

    oracle/_ref/realdataset_search is the reference's realdataset_search built from its
    sources by oracle/build_ref.sh (2 attributes on a 4x4 grid, no range override, and
    two memory-safety fixes of its planner launches).  Both binaries read the same
    reference-format files (config 2, ids renumbered cell-major, ground truth from the
    GPU exact scan) with the reference's flags --prefilter 0.0 --postfilter 17 --degree 32;
    the reference runs once per --alphas value (its fp16 scale factor; fp16 accumulation
    overflows without one), ours (garfield_b200/bin/realdataset_search) once.  Each writes
    the reference's CSV (ef, recall, qps = qnum / (cost1 + cost2 + cost3), ...).  Reported:
    both sweeps, each side's best QPS at recall >= --target, and the same with the
    search alone (qnum / cost3)."""
    import torch
    import garfield_b200 as gf
    from garfield_b200 import indexbuild
    ref = _ref_binary("realdataset_search")
    ours = ROOT / "garfield_b200" / "bin" / "realdataset_search"
    if ref is None:
        print(json.dumps({"impl": "reference-cuda", "unavailable": "oracle/_ref/realdataset_search is not built "
                          "(oracle/build_ref.sh needs the reference checkout)"}), flush=True)
        return
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    ds, ix = dataset_and_index(args, device)
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                            r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree,
                            cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, keep_fp32=True)
    gt, _ = index.bruteforce(torch.from_numpy(ds.queries).cuda(), torch.from_numpy(ds.lo.astype(np.float32)).cuda(),
                             torch.from_numpy(ds.hi.astype(np.float32)).cuda(), 10)
    gt = gt.cpu().numpy().view(np.uint32)
    index.close()
    del index
    torch.cuda.empty_cache()
    ds2, ix2, gt2 = _cell_major(ds, ix, gt)
    out_dir = Path(args.out_dir)
    d = Path(args.cache) / "ref_files"
    paths = indexbuild.write_files(d, "cfg2", ds2, ix2, gt=gt2)
    flags = ["--data_path", paths["data_path"], "--query_path", paths["query_path"], "--range", paths["range"],
             "--gt", paths["gt"], "--cagra_prefix", paths["cagra_prefix"], "--cagra_suffix", paths["cagra_suffix"],
             "--global_graph", paths["global_graph"], "--grid", paths["grid"], "--attrs", paths["attrs"],
             "--cluster", paths["cluster"], "--prefilter", "0.0", "--postfilter", "17", "--degree", str(ix.degree)]
    out_dir.mkdir(parents=True, exist_ok=True)
    runs = []
    for alpha in args.alphas:
        csv = d / f"reference_{alpha}.csv"
        csv.unlink(missing_ok=True)
        t0 = time.time()
        r = subprocess.run([str(ref)] + flags + ["--result", str(csv), "--f2h_factor", str(alpha)],
                           capture_output=True, text=True, timeout=args.ref_timeout)
        log(f"reference alpha={alpha} rc={r.returncode} in {time.time() - t0:.0f}s")
        (out_dir / f"reference_cuda_alpha{alpha}.log").write_text(
            r.stdout[-100000:] + "\n---stderr---\n" + r.stderr[-20000:])
        runs.append({"alpha": alpha, "rc": r.returncode, "rows": _read_csv(csv) if csv.exists() else []})
        if r.returncode != 0 or "illegal" in (r.stdout + r.stderr):
            log("reference run failed; not running it again")
            break
    csv = d / "ours.csv"
    csv.unlink(missing_ok=True)
    r = subprocess.run([str(ours)] + flags + ["--result", str(csv), "--f2h_factor", "1.0", "--width",
                                              str(args.width or 4)], capture_output=True, text=True, timeout=600)
    (out_dir / "ours_cli.log").write_text(r.stdout[-50000:] + "\n---stderr---\n" + r.stderr[-20000:])
    mine = _read_csv(csv) if csv.exists() else []
    ref_rows = [dict(row, alpha=run["alpha"]) for run in runs for row in run["rows"]]
    for rows in (ref_rows, mine):
        for row in rows:
            row["search_qps"] = round(args.qnum / row["cost3"], 1) if row["cost3"] > 0 else None
    best_ref, best_ours = _best(ref_rows, args.target), _best(mine, args.target)
    best_ref_s = max((r for r in ref_rows if r["recall"] >= args.target), key=lambda r: r["search_qps"] or 0,
                     default=None)
    best_ours_s = max((r for r in mine if r["recall"] >= args.target), key=lambda r: r["search_qps"] or 0,
                      default=None)
    by_ef = {}
    for row in ref_rows:
        if row["ef"] not in by_ef or row["recall"] > by_ef[row["ef"]]:
            by_ef[row["ef"]] = row["recall"]
    recall_gap = {row["ef"]: round(row["recall"] - by_ef[row["ef"]], 4) for row in mine if row["ef"] in by_ef}
    print(json.dumps({
        "impl": "reference-cuda", "metric": f"QPS at recall@10>={args.target} (1M x 128, 2 attrs, {args.sel:.0%} sel.)",
        "value": None if best_ref is None else best_ref["qps"], "unit": "queries/s",
        "ours_value": None if best_ours is None else best_ours["qps"],
        "qps_ratio": (None if not (best_ref and best_ours) else round(best_ours["qps"] / best_ref["qps"], 2)),
        "search_only_ratio": (None if not (best_ref_s and best_ours_s) else
                              round(best_ours_s["search_qps"] / best_ref_s["search_qps"], 2)),
        "best_reference": best_ref, "best_ours": best_ours, "best_reference_search_only": best_ref_s,
        "best_ours_search_only": best_ours_s, "recall_ours_minus_reference_by_ef": recall_gap,
        # north star: graph-search recall within 0.5 points of the reference's at matched L
        "recall_within_half_point": bool(recall_gap) and min(recall_gap.values()) >= -0.005,
        "reference_runs": runs, "ours_rows": mine, "qnum": int(args.qnum),
        "files": "config2, ids renumbered cell-major, ground truth = GPU exact scan",
        "flags": "--prefilter 0.0 --postfilter 17 --degree 32 (ours adds --width and --f2h_factor 1.0)"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-cuda"])
    ap.add_argument("--sel", type=float, default=None)  # default: 0.10 (config 2), 0.02 (config 4)
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5])  # data shape
    ap.add_argument("--prefilter", type=float, default=0.0)  # --prefilter: box share at or below -> exact route
    ap.add_argument("--exact-tc", dest="exact_tc", type=int, default=0)  # exact route on the tensor cores
    ap.add_argument("--route", type=int, default=0)  # 1: route each query by cost (graph or tensor-core scan)
    ap.add_argument("--target", type=float, default=0.95)
    ap.add_argument("--L", type=int, default=0)
    ap.add_argument("--width", type=int, default=0)  # 0 = pick the faster of 4 and 8
    # --points is the same flag for launchers whose own parser takes "--n" as an abbreviation
    ap.add_argument("--n", "--points", dest="n", type=int, default=1_000_000)
    ap.add_argument("--qnum", type=int, default=10_000)
    ap.add_argument("--R", type=int, default=None)  # default: 32, 64 for config 4
    ap.add_argument("--E", type=int, default=2)
    ap.add_argument("--C", type=int, default=1000)
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--gt-sample", dest="gt_sample", type=int, default=10_000)
    ap.add_argument("--cpu-sample", dest="cpu_sample", type=int, default=200)
    ap.add_argument("--ref-sample", dest="ref_sample", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", dest="no_cpu_baseline", action="store_true")
    ap.add_argument("--cache", default=str(ROOT / ".gf_cache"))  # synthetic indexes, kept out of git
    ap.add_argument("--out-dir", dest="out_dir", default=str(ROOT / ".gf_cache" / "logs"))  # --impl reference-cuda logs
    ap.add_argument("--alphas", type=float, nargs="+", default=[0.01, 0.005, 0.02])
    ap.add_argument("--ref-timeout", dest="ref_timeout", type=int, default=900)
    ap.add_argument("--mode", default="in-memory",
                    choices=["in-memory", "out-of-core", "sharded", "bruteforce", "fullgraph"])
    ap.add_argument("--batch-cells", dest="batch_cells", type=int, default=4)
    ap.add_argument("--cross-spokesman", dest="cross_spokesman", action="store_true",
                    help="keep the cross-cell edges of spokesmen only (row f2 of the scope table)")
    args = ap.parse_args()
    if args.sel is None:
        args.sel = {2: 0.10, 3: 0.05, 4: 0.02, 5: 0.01}[args.config]
    args.k = 100 if args.config == 3 else 10
    if args.route:  # routing by cost sends queries to the tensor-core exact scan
        args.exact_tc = 1
    if args.R is None:
        args.R = 64 if args.config == 4 else 32
    if args.config in (3, 4) and args.mode not in ("in-memory", "bruteforce"):
        ap.error("--config 3 and 4 apply to the in-memory and bruteforce modes")
    if args.config == 5 and args.mode not in ("out-of-core", "sharded"):
        ap.error("--config 5 applies to the out-of-core and sharded modes")
    if args.impl == "ours" and args.mode == "out-of-core":
        run_out_of_core(args)
    elif args.impl == "ours" and args.mode == "sharded":
        run_sharded(args)
    elif args.impl == "ours" and args.mode == "bruteforce":
        run_bruteforce(args)
    elif args.impl == "ours" and args.mode == "fullgraph":
        run_fullgraph(args)
    elif args.impl == "reference":
        run_reference_cpu(args)
    elif args.impl == "reference-cuda":
        run_reference_cuda(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
