"""The C-ABI library loads and exports every symbol include/*.h declares (no compute calls)."""
import ctypes as ct
import re
import subprocess
from pathlib import Path

import pytest

import appt_spgemm as ap

ROOT = Path(__file__).resolve().parent.parent


def _declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:extern\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(",
                             text, flags=re.M):
            name = m.group(1)
            if name not in ("if", "while", "for", "return", "sizeof"):
                names.add(name)
        for m in re.finditer(r"^\s*extern\s+bool\s+(\w+);", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_library_builds_and_loads():
    lib = ap.load()
    assert ap.library_path().exists()
    assert "sm_100a" in ap.version()
    assert lib is ap.load()


def test_every_declared_symbol_is_exported():
    declared = _declared_functions()
    assert {"appt_spgemm", "spgemm_self_product_adaptive", "spgemm_att_adaptive", "build_csc",
            "mempool_init", "pinned_d2h_alloc", "g_use_mempool"} <= declared
    out = subprocess.run(["nm", "-D", "--defined-only", str(ap.library_path())], check=True,
                         capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    missing = sorted(declared - exported)
    assert not missing, missing
    lib = ap.load()
    for name in declared:
        assert hasattr(lib, name), name


def test_cxx_linkage_entry_points_for_the_reference_driver():
    """The reference's src/main.cu links against the C++ (mangled) names of spgemm.h."""
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", str(ap.library_path())], check=True,
                         capture_output=True, text=True).stdout
    for sig in ("spgemm_self_product_adaptive(void*, int, int, int, void**, int*, int*, int*)",
                "spgemm_att_adaptive(void*, int, int, int, void**, int*, int*, int*)",
                "spgemm_transpose_product(void*, int, int, int, void**, int*, int*, int*)",
                "spgemm_self_product(void*, int, int, int, void**, int*, int*, int*)",
                "mempool_init(unsigned long)", "pinned_d2h_alloc(void**, unsigned long)",
                "build_csc(int const*, int const*, double const*, int, int, int**, int**, double**)",
                "should_run_method(char const*)"):
        assert sig in out, sig


def test_host_only_helpers_without_gpu(monkeypatch):
    lib = ap.load()
    monkeypatch.setenv("METHOD", "hash")
    assert lib.should_run_method(b"HASH")
    assert not lib.should_run_method(b"merge3")
    monkeypatch.setenv("METHOD", "all")
    assert lib.should_run_method(b"anything")
    import numpy as np
    from appt_spgemm import matrices as M
    import oracle
    A = M.uniform8(n=512)
    assert abs(ap.reference_score(A) - oracle.reference_score(A)) < 1e-12
    o = ap.Options()
    lib.appt_default_options(ct.byref(o))
    assert (o.op, o.method, o.in_mem, o.out_mem, o.device) == (0, 0, 0, 0, 0)
