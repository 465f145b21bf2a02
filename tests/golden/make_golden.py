"""Generate the golden fixtures in this directory from the reference itself.

Run in a container that has the reference checkout (path as the first argument);
the GPU box never runs this script, it only reads the .npz files it writes.

  golden_grid.npz     the reference's own grid_scatter_V2 (indexbuild/tools.py:88-125),
                      executed from its source: the module imports cupy/cuvs at the top,
                      so the function definitions are extracted with `ast` and run with numpy
  golden_bf.npz       naive_brute_force_with_filter (gpu_graph.cu:10782-10812) run on the CPU
                      by oracle/_ref/ref_golden (built from the reference's sources by
                      `make -C oracle ref_golden REF=<checkout>`)
  golden_cluster.npz  load_clustering (tools.cuh:569-602) run the same way: centroids and
                      the cell x cluster histogram (cells = i / 62500 in the reference)
  golden_quant.npz    the reference's host int8 quantiser (production_adapter.cuh:316-337,
                      via load_dataset_return_int8_arr_infile) run the same way: the .q file
                      it writes (codes, scales, zero points)
  golden_spokesman.npz the reference's cross-graph compression compress_global_graph_extreme
                      and its writer save_global_graph_extreme (tools.cuh:917-1038) run on the
                      CPU by oracle/_ref/ref_spokesman (`make -C oracle ref_spokesman REF=...`):
                      the compressed-graph file it writes, for seeded per-cell graphs

Inputs are seeded synthetic arrays written next to the outputs.
"""
from __future__ import annotations

import ast
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def load_reference_functions(ref: Path, names: list[str]) -> dict:
    src = (ref / "indexbuild" / "tools.py").read_text()
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    mod = ast.Module(body=keep, type_ignores=[])
    ns: dict = {"np": np, "print": lambda *a, **k: None}
    exec(compile(mod, str(ref / "indexbuild" / "tools.py"), "exec"), ns)
    return ns


def golden_grid(ref: Path) -> None:
    ns = load_reference_functions(ref, ["grid_scatter_V2"])
    rng = np.random.default_rng(20261201)
    cases = {}
    # ties across slice boundaries, a non-divisible n, 1-3 dimensions
    for name, n, grid, hi in [("a", 1000, [4, 4], 100), ("b", 997, [3, 5], 10000), ("c", 640, [2, 2, 2], 7),
                              ("d", 400, [8], 1000)]:
        attrs = rng.integers(0, hi, size=(n, len(grid))).astype(np.int32)
        p_infos, gpid = ns["grid_scatter_V2"](attrs, np.array(grid, np.int32))
        cases[f"{name}_attrs"] = attrs
        cases[f"{name}_grid"] = np.array(grid, np.int32)
        cases[f"{name}_lq"] = np.concatenate([np.asarray(p[0]) for p in p_infos]).astype(np.int32)
        cases[f"{name}_rq"] = np.concatenate([np.asarray(p[1]) for p in p_infos]).astype(np.int32)
        cases[f"{name}_slices"] = np.stack([np.asarray(p[2]) for p in p_infos], 1).astype(np.int32)
        cases[f"{name}_gpid"] = np.asarray(gpid, np.int32)
    np.savez_compressed(HERE / "golden_grid.npz", **cases)


def golden_bf_and_cluster(ref_bin: Path) -> None:
    import garfield_b200 as gf
    from garfield_b200 import synth
    ds = synth.make(3000, 32, 20, 40, (2, 2), 0.2, domain=1000, seed=77, stratified=False)
    # a few exact duplicates and equal-distance points to exercise ties (lower id wins)
    ds.vectors[100] = ds.vectors[50]
    ds.vectors[2000] = ds.vectors[50]
    ds.attrs[100] = ds.attrs[50]
    ds.attrs[2000] = ds.attrs[50]
    ds.queries[0] = ds.vectors[50]
    ds.lo[0] = ds.attrs[50] - 5
    ds.hi[0] = ds.attrs[50] + 5
    k = 10
    labels = np.random.default_rng(5).integers(0, 12, size=3000).astype(np.int32)
    with tempfile.TemporaryDirectory() as td:
        t = Path(td)
        gf.write_fvecs(t / "d.fvecs", ds.vectors)
        gf.write_attrs(t / "a.attrs", ds.attrs)
        gf.write_fvecs(t / "q.fvecs", ds.queries)
        gf.write_ranges(t / "r.range", ds.lo, ds.hi)
        subprocess.run([str(ref_bin), "bf", str(t / "d.fvecs"), str(t / "a.attrs"), str(t / "q.fvecs"),
                        str(t / "r.range"), str(k), str(t / "bf.u32")], check=True, capture_output=True)
        bf = np.fromfile(t / "bf.u32", np.uint32).reshape(len(ds.queries), k)
        with open(t / "c.bin", "wb") as f:
            f.write(np.array([len(labels)], np.int32).tobytes() + labels.tobytes())
        subprocess.run([str(ref_bin), "cluster", str(t / "d.fvecs"), str(t / "c.bin"), str(t / "cent.f32"),
                        str(t / "hist.u32")], check=True, capture_output=True)
        cent = np.fromfile(t / "cent.f32", np.float32).reshape(-1, ds.vectors.shape[1])
        hist = np.fromfile(t / "hist.u32", np.uint32).reshape(16, -1)
    np.savez_compressed(HERE / "golden_bf.npz", vectors=ds.vectors, attrs=ds.attrs, queries=ds.queries, lo=ds.lo,
                        hi=ds.hi, ids_heap_order=bf, k=np.int32(k))
    np.savez_compressed(HERE / "golden_cluster.npz", labels=labels, centroids=cent, hist=hist)


def golden_quant(ref_bin: Path) -> None:
    import garfield_b200 as gf
    rng = np.random.default_rng(31)
    # mixture-like data in [0, 255] with a clipped tail, a constant-free set of dimensions,
    # values on rounding boundaries, and a negative range (zero point clamping)
    x = np.clip(rng.normal(100, 40, size=(700, 24)), 0, 255).astype(np.float32)
    x[:, 3] = rng.integers(0, 256, size=700).astype(np.float32)
    x[:, 5] = np.round(x[:, 5]) + 0.5
    x[:, 7] = -x[:, 7] - 10.0
    out = {}
    with tempfile.TemporaryDirectory() as td:
        t = Path(td)
        gf.write_fvecs(t / "d.fvecs", x)
        for name, alpha in (("a1", 1.0), ("a05", 0.5), ("a3", 3.0)):
            qpath = t / f"{name}.q"
            subprocess.run([str(ref_bin), "quant", str(t / "d.fvecs"), repr(alpha), str(qpath)], check=True,
                           capture_output=True)
            codes, sc, zp = gf.read_q(qpath)
            out[f"{name}_codes"], out[f"{name}_scales"], out[f"{name}_zps"] = codes, sc, zp
            out[f"{name}_alpha"] = np.float32(alpha)
    np.savez_compressed(HERE / "golden_quant.npz", data=x, **out)


def golden_spokesman(ref_bin: Path) -> None:
    rng = np.random.default_rng(20261207)
    sizes = np.array([700, 500, 650, 400, 3], np.uint32)
    R, E = 8, 2
    n, P = int(sizes.sum()), len(sizes)
    graphs = np.concatenate([rng.integers(0, s, size=(s, R)) for s in sizes]).astype(np.uint32)
    cross_t = np.stack([rng.integers(0, sizes[c], size=(n, E)) for c in range(P)]).astype(np.uint32)
    with tempfile.TemporaryDirectory() as td:
        t = Path(td)
        graphs.tofile(t / "g.u32")
        sizes.tofile(t / "s.u32")
        cross_t.tofile(t / "x.u32")
        subprocess.run([str(ref_bin), str(t / "g.u32"), str(t / "s.u32"), str(t / "x.u32"), str(R), str(E),
                        str(t / "out.bin")], check=True, capture_output=True)
        raw = np.fromfile(t / "out.bin", np.uint32)
    hn, hp, he = (int(v) for v in raw[:3])
    cn = raw[3:3 + hp]
    co = raw[3 + hp:3 + 2 * hp]
    cp = raw[3 + 2 * hp:3 + 2 * hp + hn]
    edges = raw[3 + 2 * hp + hn:].reshape(hp, int(cn.sum()), he)
    np.savez_compressed(HERE / "golden_spokesman.npz", sizes=sizes, graphs=graphs, cross_t=cross_t, degree=R, e=E,
                        center_num=cn, col_offset=co, center_pos=cp, edges=edges, raw=raw)


def main() -> None:
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 else None
    if ref is None or not (ref / "indexbuild" / "tools.py").exists():
        raise SystemExit("usage: make_golden.py <reference checkout>")
    golden_grid(ref)
    ref_bin = ROOT / "oracle" / "_ref" / "ref_golden"
    if not ref_bin.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "ref_golden", f"REF={ref}"], check=True)
    golden_bf_and_cluster(ref_bin)
    golden_quant(ref_bin)
    spk_bin = ROOT / "oracle" / "_ref" / "ref_spokesman"
    if not spk_bin.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "ref_spokesman", f"REF={ref}"], check=True)
    golden_spokesman(spk_bin)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
