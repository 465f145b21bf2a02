"""Build libgarfield_b200.so and the realdataset_search CLI for sm_100a with nvcc.

Objects go to _build/ at the repository root; the shared library and the CLI are
written in-tree (garfield_b200/libgarfield_b200.so, garfield_b200/bin/) so they travel
with the source tree.  Rebuilds only what changed (mtime check against sources and
headers).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libgarfield_b200.so"
BIN = PKG / "bin"

LIB_SOURCES = ["gf_index.cu", "gf_io.cpp", "gf_plan.cu", "gf_search.cu", "gf_bruteforce.cu", "gf_noalloc.cu", "gf_batch.cu", "gf_schedule.cpp", "gf_codec.cu", "gf_centroid_tc.cu", "gf_bf_tc.cu"]
CLI_SOURCES = ["gf_cli.cpp"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
          "--expt-relaxed-constexpr", "-Xcompiler", "-Wall,-Wno-unused-function"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [INCLUDE / "garfield.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, flush=True)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    BIN.mkdir(exist_ok=True)
    headers = _headers()
    objs = []
    jobs = []
    for name in LIB_SOURCES + CLI_SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if ptxas_info:
        COMMON.extend(["-Xptxas", "-v"])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for f in [ex.submit(_compile, s, o, verbose or ptxas_info) for s, o in jobs]:
            f.result()
    lib_objs = [BUILD / (n + ".o") for n in LIB_SOURCES]
    if _stale(LIB, lib_objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, lib_objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    cli = BIN / "realdataset_search"
    cli_objs = [BUILD / (n + ".o") for n in CLI_SOURCES]
    if _stale(cli, cli_objs + [LIB]):
        cmd = [nvcc(), *ARCH, "-cudart", "static", "-o", str(cli), *map(str, cli_objs), "-L", str(PKG),
               "-lgarfield_b200", "-Xlinker", "-rpath,$ORIGIN/.."]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"CLI link failed:\n{r.stdout}\n{r.stderr}")
        normal = BIN / "normaldataset_search"
        if normal.exists() or normal.is_symlink():
            normal.unlink()
        normal.symlink_to("realdataset_search")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(f"built {LIB}")
