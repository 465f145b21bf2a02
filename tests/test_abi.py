"""The C ABI library loads without a GPU and exports every function include/garfield.h declares."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import garfield_b200 as gf

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "garfield.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gf_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_all():
    lib = gf.lib()
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(gf.lib_path)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (gf_[a-z0-9_]+)", out))
    assert set(names) <= exported


def test_static_strings_without_gpu():
    lib = gf.lib()
    assert b"sm_100a" in lib.gf_version()
    assert lib.gf_status_string(0) == b"ok"
    assert lib.gf_status_string(5) == b"cuda error"
    p = gf._SearchParams()
    lib.gf_search_defaults(ctypes.byref(p))
    assert (p.L, p.k, p.width, p.max_iter) == (64, 10, 1, 10000)


def test_cli_built():
    cli = ROOT / "garfield_b200" / "bin" / "realdataset_search"
    assert cli.exists()
    r = subprocess.run([str(cli)], capture_output=True, text=True)
    assert r.returncode == 2 and "--data_path" in r.stderr
