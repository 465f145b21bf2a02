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
  python bench.py --impl reference                          CPU exact filtered scan (the
                                                            oracle's restatement of the
                                                            reference's CPU path) on host cores
  python bench.py --mode out-of-core [--batch-cells B]     graphs in pinned host memory, streamed
                                                            per scheduled batch of B cells (row a17)
  torchrun ... bench.py --mode sharded                     cell-sharded index over the ranks, keys
                                                            all-gathered over NCCL and merged (row e)
  python bench.py --mode bruteforce                        exact filtered k-NN of all queries: tensor-core
                                                            pass vs the CUDA-core kernel
  python bench.py --impl reference-cuda                     the reference's own CUDA binary: prints
                                                            "unavailable" (it faults on B200, see
                                                            REF_CUDA_FAULT)
Multi-GPU (torchrun): every rank holds a replica of the index and runs the full query
batch (weak scaling); the only collective is the max-over-ranks of the timings.
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


def ncu_traffic() -> float | None:
    """DRAM bytes of one search launch from the committed ncu summary (None if absent)."""
    import re
    p = ROOT / "profiles" / "gmg_search_kernel_config2.md"
    if p.exists():
        m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", p.read_text())
        if m:
            return float(m.group(1))
    return None


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
    else:
        ds = synth.config2(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
    log(f"dataset {ds.vectors.shape} in {time.time() - t0:.1f}s")
    key = f"cfg{args.config}_n{args.n}_s{args.seed}_R{args.R}_E{args.E}_C{args.C}.npz"
    cache = Path(args.cache) / key if args.cache else None
    if cache is not None and cache.exists():
        z = np.load(cache)
        ix = indexbuild.GmgArrays(z["grid"], z["l_quant"], z["r_quant"], z["slices"], z["cell_of"], z["graphs"],
                                  z["cross"], z["labels"], int(z["degree"]), int(z["cross_e"]))
        log(f"index loaded from {cache}")
    else:
        t0 = time.time()
        ix = indexbuild.build(ds.vectors, ds.attrs, ds.grid, R=args.R, E=args.E, C=args.C, seed=args.seed,
                              device=device)
        torch.cuda.synchronize()
        log(f"index built in {time.time() - t0:.1f}s")
        if cache is not None:
            try:
                cache.parent.mkdir(parents=True, exist_ok=True)
                tmp = cache.with_suffix(f".{os.getpid()}.tmp.npz")
                np.savez(tmp, grid=ix.grid, l_quant=ix.l_quant, r_quant=ix.r_quant, slices=ix.slices,
                         cell_of=ix.cell_of, graphs=ix.graphs, cross=ix.cross, labels=ix.labels,
                         degree=ix.degree, cross_e=ix.cross_e)
                os.replace(tmp, cache)
            except OSError:
                pass
    return ds, ix


def cpu_baseline(ds, sample: int, threads: int, k: int = 10) -> dict:
    """The oracle's exact filtered scan (naive_brute_force_with_filter restated) on host cores."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    q = ds.queries[:sample]
    oracle.bruteforce(ds.vectors, ds.attrs, q[:4], ds.lo[:4], ds.hi[:4], k, threads)  # warm
    t0 = time.perf_counter()
    oracle.bruteforce(ds.vectors, ds.attrs, q, ds.lo[:sample], ds.hi[:sample], k, threads)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"{sample} queries, exact filtered scan over all {ds.vectors.shape[0]} points "
                      f"({dt:.1f}s)"}


# --------------------------------------------------------------------------- arms

def run_ours(args):
    import torch
    import torch.distributed as dist
    import garfield_b200 as gf

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    ds, ix = dataset_and_index(args, device)
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
        return gf.SearchParams(L=L, k=K, width=width, exact_tc=args.exact_tc)

    def step(L, width):
        plan.build(qd, lod, hid, args.prefilter, stream)
        plan.search(sp(L, width), stream, ids=ids, dist=dist_t)

    def find_L(width):
        """Smallest L of the sweep whose recall reaches the target at this width."""
        sweep = []
        for L in ([args.L] if args.L else [x for x in L_SWEEP if x >= K]):
            with torch.cuda.stream(stream):
                step(L, width)
            stream.synchronize()
            r = gf.recall(ids[:S].cpu().numpy().view(np.uint32), gt)
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
        return a.elapsed_time(b) / n

    widths = [args.width] if args.width else [1, 2, 4, 8]
    best = None
    for wd in widths:
        L_w, r_w, sw = find_L(wd)
        ms = quick_ms(L_w, wd) if r_w >= args.target or len(widths) == 1 else float("inf")
        log(f"width={wd}: L={L_w} recall={r_w:.4f} {ms:.3f} ms/step")
        if best is None or ms < best[3]:
            best = (wd, L_w, r_w, ms, sw)
    args.width, L, recall, _, sweep = best
    # L2 flush buffer (> 126 MB L2)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            step(L, args.width)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(float(i))
                ev[i][0].record(stream)
                plan.build(qd, lod, hid, args.prefilter, stream)
                ev[i][1].record(stream)
                plan.search(sp(L, args.width), stream, ids=ids, dist=dist_t)
                ev[i][2].record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    step_ms = [a.elapsed_time(c) for a, b, c in ev]
    plan_ms = [a.elapsed_time(b) for a, b, c in ev]
    search_ms = [b.elapsed_time(c) for a, b, c in ev]
    st = plan.stats()
    total_ms = float(sum(step_ms))
    if world > 1:
        t = torch.tensor([total_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
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
    e2e_total = float(sum(e_ms))
    if world > 1:
        t = torch.tensor([e2e_total], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_total = float(t.item())
    e2e_value = world * qnum / (e2e_total / args.steps / 1e3)
    assert np.array_equal(res_ids, ids.cpu().numpy().view(np.uint32))
    # roofline of the search kernel: algorithmic bytes from the device counters
    D, a_attr = ds.vectors.shape[1], ds.attrs.shape[1]
    bytes_step = (st["n_dist"] * (((D + 7) // 8 * 8) * 2 + a_attr * 4) + st["n_exp"] * ix.degree * 4 +
                  st["n_cross"] * (ix.cross_e * 4 + (4 if args.cross_spokesman else 0)))
    kern_s = float(np.mean(search_ms)) / 1e3
    achieved = bytes_step / kern_s / 1e9
    peak, peak_kind = peak_hbm()
    out = {
        "metric": f"QPS at recall@{K}>={args.target} ({SHAPES[args.config].format(sel=args.sel)})",
        "value": round(value, 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 accumulate",
        "data": f"synthetic (seeded Gaussian mixture; BASELINE config {args.config} shapes)",
        "config": {"workload": (f"config{args.config}: {ds.vectors.shape[0]} x {D} fp32, grid "
                                f"{'x'.join(str(int(g)) for g in ix.grid)}, R={ix.degree}, E={ix.cross_e}, C={args.C}, "
                                f"{qnum} queries, sel {args.sel:.0%}, k={K}"),
                   "L": L, "width": args.width, f"recall_at_{K}": round(recall, 4), "recall_sample": S,
                   "l2": "flushed (256 MiB write) between timed steps", "parallelism": f"replicas x{world}",
                   "plan_ms": round(float(np.mean(plan_ms)), 4), "search_ms": round(float(np.mean(search_ms)), 4),
                   "prefilter": args.prefilter, "exact_route": ("tensor-core exact scan" if args.exact_tc
                                                                else "fp16 warp scan"), "n_exact": int(st["n_exact"]),
                   "sweep": sweep,
                   "cross_edges": (f"spokesman rows only: {index.cross_rows} of {index.n} (compress_global_graph_extreme)"
                                   if args.cross_spokesman else "full")},
        "e2e": {"value": round(e2e_value, 1), "unit": "queries/s",
                "h2d_bytes_per_step": int(qh.nbytes + lh.nbytes + hh.nbytes), "d2h_bytes_per_step": int(qnum * K * 4)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": ncu_traffic(),
                     "kernel": "gmg_search_kernel", "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": int(bytes_step),
                     "counters": {k: int(v) for k, v in st.items()}},
        "clocks": clocks.summary(),
        # per step: f2h, cell count, cell fill, centroid top-4, centroid merge, cell order, iota,
        # search (the CUB scan and radix-sort kernels of the planner are library launches)
        "gpu_launches": 8 * args.steps,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(ds, args.cpu_sample, os.cpu_count() or 1, K)
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
    streamed = gf.Index.create(**common, keep_fp32=True, host_graph=True)
    resident = gf.Index.create(**common, keep_fp32=False, host_graph=False)
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
        seg = np.bincount(ix.cell_of, minlength=int(np.prod(ix.grid)))
        h2d = sum(int(seg[c]) * ix.degree * 4 + len(bt) * int(seg[c]) * ix.cross_e * 4 for bt in batches for c in bt)
        res[name] = {"qps": round(qnum / (float(np.mean(ms)) / 1e3), 1), "ms_per_step": round(float(np.mean(ms)), 4),
                     "L": L, "recall_at_10": round(recall, 4), "sweep": sweep,
                     "h2d_graph_bytes_per_step": h2d if name == "streamed" else 0}
        res["batches"], res["splits"], res["schedule_ms"] = batches, splits, round(sched_ms, 3)
        plan.close()
    out = {"metric": "QPS at recall@10>=0.95, graphs streamed per batch of cells (1M x 128, 2 attrs, 10% sel.)",
           "value": res["streamed"]["qps"], "unit": "queries/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": res["streamed"]["ms_per_step"], "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 accumulate",
           "data": "synthetic (seeded Gaussian mixture; BASELINE config 2 shapes)",
           "config": {"workload": "config2, out-of-core batches", "batch_cells": args.batch_cells, "width": width,
                      "n_batches": len(res["batches"]), "splits": res["splits"], "schedule_ms": res["schedule_ms"],
                      "batches": res["batches"], "streamed": res["streamed"], "resident_same_batches": res["resident"],
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
    """Exact filtered k-NN mode (gf_bruteforce, the GPU ground truth): config-2 data, all 10k
    queries, k = 10.  Times the tensor-core pass (query x point products on tcgen05 with a
    proven error bound, exact re-rank, CUDA-core answer for unproven queries) beside the
    CUDA-core kernel on the same inputs, and checks that both return the same ids and
    distances.  The roofline is the tensor pipe: executed MMA FLOPs per second."""
    import torch
    import garfield_b200 as gf
    from garfield_b200 import indexbuild, synth
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    K = args.k
    if args.config == 3:
        ds = synth.config3(seed=args.seed, n=args.n, qnum=args.qnum, n_centers=max(10, args.n // 1000),
                           selectivity=args.sel)
        shape = f"{args.n // 10**6}M x 96 unit-norm, 3 attrs on 4x4x4, {args.sel:.0%} sel., k=100"
    elif args.config == 4:
        ds = synth.config4(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
        shape = f"{args.n // 10**6}M x 768 unit-norm, 2 attrs on 8x8, {args.sel:.0%} sel., k=10"
    else:
        ds = synth.config2(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
        shape = f"{args.n // 10**6}M x 128, 2 attrs, {args.sel:.0%} sel., k=10"
    lq, rq, _, cell_of = indexbuild.quantile_grid(ds.attrs, ds.grid)
    n, D = ds.vectors.shape
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=np.asarray(ds.grid, np.uint32),
                            l_quant=lq, r_quant=rq, cell_of=cell_of, graphs=np.zeros((n, 1), np.uint32), degree=1,
                            keep_fp32=True, device=local)
    qnum = ds.queries.shape[0]
    qd = torch.from_numpy(ds.queries).to(device)
    lod = torch.from_numpy(ds.lo.astype(np.float32)).to(device)
    hid = torch.from_numpy(ds.hi.astype(np.float32)).to(device)
    stream = torch.cuda.Stream(device)
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=device)
    stats = torch.zeros(3, dtype=torch.int32, device=device)

    def timed(path, steps, warmup):
        for _ in range(warmup):
            index.bruteforce(qd, lod, hid, K, stream=stream, path=path, stats=stats)
        stream.synchronize()
        ms = []
        with ClockSampler(local) as clocks:
            for i in range(steps):
                with torch.cuda.stream(stream):
                    flush.fill_(float(i))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                ids, dist = index.bruteforce(qd, lod, hid, K, stream=stream, path=path, stats=stats)
                b.record(stream)
                b.synchronize()
                ms.append(a.elapsed_time(b))
        return ids, dist, float(np.mean(ms)), stats.cpu().numpy().copy(), clocks.summary()

    t_ids, t_d, t_ms, st, clocks = timed(2, args.steps, args.warmup)
    c_ids, c_d, c_ms, _, _ = timed(1, 1, 1)
    same = bool(torch.equal(t_ids, c_ids) and torch.equal(t_d, c_d))
    # end to end: host queries and boxes in pinned memory, ids back to the host
    qh, lh, hh = (torch.from_numpy(x).pin_memory() for x in (ds.queries, ds.lo.astype(np.float32),
                                                              ds.hi.astype(np.float32)))
    qg, lg, hg = torch.empty_like(qd), torch.empty_like(lod), torch.empty_like(hid)
    ih = torch.empty((qnum, K), dtype=torch.int32).pin_memory()
    e_ms = []
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
    products = int(st[2])
    dp = (D + 15) // 16 * 16
    flops = 2.0 * products * 128 * 128 * dp
    achieved = flops / (t_ms / 1e3) / 1e12
    peak, peak_kind = peak_tensor()
    out = {"metric": f"exact filtered k-NN queries/s ({shape})",
           "value": round(qnum / (t_ms / 1e3), 1), "unit": "queries/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(t_ms, 4), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f16 products, f32 accumulate, f32 exact re-rank",
           "data": f"synthetic (seeded Gaussian mixture; BASELINE config {args.config} shapes)",
           "config": {"workload": f"config{args.config} brute force: {n} x {D} fp32, {qnum} queries, "
                                  f"sel {args.sel:.0%}, k={K}",
                      "l2": "flushed (256 MiB write) between timed steps",
                      "cuda_core_ms_per_step": round(c_ms, 3), "speedup_vs_cuda_cores": round(c_ms / t_ms, 2),
                      "identical_to_cuda_cores": same, "fallback_queries": int(st[0]), "timeouts": int(st[1]),
                      "tile_products": products, "dense_products": ((qnum + 127) // 128) * ((n + 127) // 128)},
           "e2e": {"value": round(qnum / (float(np.mean(e_ms)) / 1e3), 1), "unit": "queries/s",
                   "h2d_bytes_per_step": int(qh.nbytes + lh.nbytes + hh.nbytes), "d2h_bytes_per_step": int(ih.nbytes)},
           "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(achieved / peak, 4), "traffic": None, "kernel": "bf_tc_kernel (whole call timed)",
                        "peak_kind": peak_kind, "flops_per_step": flops},
           "clocks": clocks,
           # morton, 3 radix-sort passes are CUB's; prep, boxes, tiles, tc, merge, CUDA-core list
           "gpu_launches": 6 * args.steps}
    if not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(ds, args.cpu_sample, os.cpu_count() or 1, K)
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
    dist.shard_cells(grid, N)[r] only; a step plans all queries on every rank, searches them
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
    index = gf.Index.create(vectors=ds.vectors, attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                            r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree,
                            cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, f2h_factor=1.0, keep_fp32=False,
                            shard_cells=mine if world > 1 else None, device=local)
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
        whole = gf.Index.create(vectors=ds.vectors,
                                attrs=ds.attrs.astype(np.float32), grid=ix.grid, l_quant=ix.l_quant,
                                r_quant=ix.r_quant, cell_of=ix.cell_of, graphs=ix.graphs, degree=ix.degree,
                                cross=ix.cross, cross_e=ix.cross_e, labels=ix.labels, keep_fp32=True, device=local)
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
    out = {"metric": "QPS at recall@10>=0.95, cell-sharded index (1M x 128, 2 attrs, 10% sel.)",
           "value": round(qnum / (ms / 1e3), 1), "unit": "queries/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "f16 storage, f32 accumulate",
           "data": "synthetic (seeded Gaussian mixture; BASELINE config 2 shapes)",
           "config": {"workload": "config2, cell-sharded", "parallelism": f"cell shards x{world}", "L": L,
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


def run_reference_cpu(args):
    """Reference arm: the CPU exact filtered scan on the host cores, same metric/config."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    from garfield_b200 import synth
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    ds = synth.config2(seed=args.seed, selectivity=args.sel, n=args.n, qnum=args.qnum)
    threads = os.cpu_count() or 1
    S = args.ref_sample
    oracle.bruteforce(ds.vectors, ds.attrs, ds.queries[:2], ds.lo[:2], ds.hi[:2], 10, threads)
    times = []
    for i in range(args.warmup + args.steps):
        s0 = (i * S) % max(1, ds.queries.shape[0] - S)
        t0 = time.perf_counter()
        oracle.bruteforce(ds.vectors, ds.attrs, ds.queries[s0:s0 + S], ds.lo[s0:s0 + S], ds.hi[s0:s0 + S], 10,
                          threads)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    value = S / float(np.mean(times))
    out = {
        "impl": "reference", "metric": "QPS at recall@10>=0.95 (1M x 128, 2 attrs, 10% sel.)",
        "value": round(value, 2), "unit": "queries/s", "n_gpus": int(os.environ.get("WORLD_SIZE", 1)),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(float(np.mean(times)) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian mixture; BASELINE config 2 shapes)",
        "config": {"workload": "config2: 1M x 128 fp32, 2 attrs, 10k queries, sel 10%, k=10",
                   "step": f"{S} queries (bounded sample), exact scan (recall 1.0)"},
        "cpu_baseline": {"value": round(value, 2), "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"{S} queries per step, exact filtered scan over {ds.vectors.shape[0]} points"},
        "e2e": {"value": round(value, 2), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


REF_CUDA_FAULT = (
    "the reference's realdataset_search (built from source for sm_100a) raised an illegal memory access on "
    "B200: prefiltering_tag_elements is launched <<<qnum, 32>>> without dynamic shared memory "
    "(real_dataset_adapter.cuh:501) but writes the query box into extern __shared__ memory (:348-353); "
    "not run again")


def run_reference_cuda(args):
    """The reference's own CUDA search: not run (it faults on this GPU, see REF_CUDA_FAULT)."""
    print(json.dumps({"impl": "reference-cuda", "unavailable": REF_CUDA_FAULT}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-cuda"])
    ap.add_argument("--sel", type=float, default=None)  # default: 0.10 (config 2), 0.02 (config 4)
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4])  # data shape (in-memory, bruteforce)
    ap.add_argument("--prefilter", type=float, default=0.0)  # --prefilter: box share at or below -> exact route
    ap.add_argument("--exact-tc", dest="exact_tc", type=int, default=0)  # exact route on the tensor cores
    ap.add_argument("--target", type=float, default=0.95)
    ap.add_argument("--L", type=int, default=0)
    ap.add_argument("--width", type=int, default=0)  # 0 = pick the fastest of 1, 2, 4, 8
    ap.add_argument("--n", type=int, default=1_000_000)
    ap.add_argument("--qnum", type=int, default=10_000)
    ap.add_argument("--R", type=int, default=None)  # default: 32, 64 for config 4
    ap.add_argument("--E", type=int, default=2)
    ap.add_argument("--C", type=int, default=1000)
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--gt-sample", dest="gt_sample", type=int, default=10_000)
    ap.add_argument("--cpu-sample", dest="cpu_sample", type=int, default=200)
    ap.add_argument("--ref-sample", dest="ref_sample", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", dest="no_cpu_baseline", action="store_true")
    ap.add_argument("--cache", default="/tmp/gf_cache")
    ap.add_argument("--alphas", type=float, nargs="+", default=[0.01])
    ap.add_argument("--ref-timeout", dest="ref_timeout", type=int, default=900)
    ap.add_argument("--mode", default="in-memory",
                    choices=["in-memory", "out-of-core", "sharded", "bruteforce", "fullgraph"])
    ap.add_argument("--batch-cells", dest="batch_cells", type=int, default=4)
    ap.add_argument("--cross-spokesman", dest="cross_spokesman", action="store_true",
                    help="keep the cross-cell edges of spokesmen only (row f2 of the scope table)")
    args = ap.parse_args()
    if args.sel is None:
        args.sel = {2: 0.10, 3: 0.05, 4: 0.02}[args.config]
    args.k = 100 if args.config == 3 else 10
    if args.R is None:
        args.R = 64 if args.config == 4 else 32
    if args.config != 2 and args.mode not in ("in-memory", "bruteforce"):
        ap.error("--config 3 and 4 apply to the in-memory and bruteforce modes")
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
