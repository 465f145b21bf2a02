"""The drop-in CLI end to end: reference-format files on disk, the binaries run with the
reference's flags (realdataset_search.cu:2712-2751), the result CSV read back
(realdataset_search.cu:2440, 2503-2509: ef,recall,qps,total_cost,cost1,cost2,cost3,
kernal_cost).  Each row's recall must be the recall of the library's own search at that
L on the same queries (the CLI is a thin wrapper over the C ABI), and QPS must be
qnum / (cost1 + cost2 + cost3)."""
from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest

import garfield_b200 as gf
import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

BIN = Path(gf.__file__).resolve().parent / "bin"


def _read_csv(path):
    lines = Path(path).read_text().strip().splitlines()
    assert lines[0] == "ef,recall,qps,total_cost,cost1,cost2,cost3,kernal_cost"
    return [[float(x) for x in line.split(",")] for line in lines[1:]]


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


@pytest.fixture(scope="module")
def files(small, tmp_path_factory):
    from garfield_b200 import indexbuild
    d = tmp_path_factory.mktemp("cli")
    return indexbuild.write_files(d, "small", small.ds, small.ix, gt=small.gt)


def _flags(paths, degree):
    return ["--data_path", paths["data_path"], "--query_path", paths["query_path"], "--range", paths["range"],
            "--gt", paths["gt"], "--cagra_prefix", paths["cagra_prefix"], "--cagra_suffix", paths["cagra_suffix"],
            "--global_graph", paths["global_graph"], "--grid", paths["grid"], "--attrs", paths["attrs"],
            "--cluster", paths["cluster"], "--prefilter", "0.0", "--postfilter", "17", "--degree", str(degree),
            "--f2h_factor", "1.0"]


def _library_recall(c, L, width):
    g = gf.Index.create(vectors=c.ds.vectors, attrs=c.ds.attrs.astype(np.float32), grid=c.ix.grid,
                        l_quant=c.ix.l_quant, r_quant=c.ix.r_quant, cell_of=c.ix.cell_of, graphs=c.ix.graphs,
                        degree=c.ix.degree, cross=c.ix.cross, cross_e=c.ix.cross_e, labels=c.ix.labels)
    ids, _ = g.search(_dev(c.ds.queries), _dev(c.ds.lo), _dev(c.ds.hi), gf.SearchParams(L=L, k=10, width=width))
    r = oracle.recall(ids.cpu().numpy().view(np.uint32), c.gt)
    g.close()
    return r


@pytest.mark.parametrize("width", [1, 4])
def test_realdataset_search_csv(small, files, tmp_path, width):
    out = tmp_path / "result.csv"
    r = subprocess.run([str(BIN / "realdataset_search")] + _flags(files, small.ix.degree) +
                       ["--result", str(out), "--ef", "16,32,64", "--width", str(width)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    rows = _read_csv(out)
    assert [int(x[0]) for x in rows] == [16, 32, 64]
    qnum = small.ds.queries.shape[0]
    for ef, recall, qps, total, c1, c2, c3, kern in rows:
        assert abs(recall - _library_recall(small, int(ef), width)) < 2e-6
        assert abs(total - (c1 + c2 + c3)) < 3e-6 and c3 > 0 and kern == c3
        # the CSV rounds total to 1 us (%.6f seconds) and qps to 1e-3
        assert abs(qps * total - qnum) <= qps * 1e-6 + 1e-2
    assert rows[-1][1] >= 0.9


def test_reference_sweep_and_normaldataset_uniform_grid(small, files, tmp_path):
    """No --ef: the reference's 33-value sweep (rows with L < k skipped).  Invoked as
    normaldataset_search the grid is uniform (--shape over [--domain_lo, --domain_hi)),
    the --grid file is ignored; the small fixture's quantile grid is the uniform 2x2 grid
    over [0, 10000), so both binaries must give the same recall at every L."""
    out_r, out_n = tmp_path / "real.csv", tmp_path / "normal.csv"
    r = subprocess.run([str(BIN / "realdataset_search")] + _flags(files, small.ix.degree) + ["--result", str(out_r)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    flags = _flags(files, small.ix.degree)
    i = flags.index("--grid")
    flags[i + 1] = str(tmp_path / "missing.grid")
    n = subprocess.run([str(BIN / "normaldataset_search")] + flags +
                       ["--result", str(out_n), "--shape", "2,2", "--domain_lo", "0", "--domain_hi", "10000"],
                       capture_output=True, text=True, timeout=600)
    assert n.returncode == 0, n.stderr[-2000:]
    real, normal = _read_csv(out_r), _read_csv(out_n)
    sweep = [10, 10, 15, 20, 25, 30, 35, 40, 45, 50, 55, 60, 70, 80, 90, 100, 120, 140, 160, 180, 200, 250, 300, 400,
             500, 600, 700, 800, 900, 1000, 1100, 1400, 1700]
    assert [int(x[0]) for x in real] == sweep and [int(x[0]) for x in normal] == sweep
    assert [x[1] for x in real] == [x[1] for x in normal]
    rec = [x[1] for x in real]
    assert rec[-1] >= 0.99 and rec[-1] >= rec[0]
