"""Build libappt_spgemm.so (sm_100a) in-tree with nvcc.

Usage: python appt-spgemm-challenge_b200/build.py [--force] [--verbose]

Objects go to appt-spgemm-challenge_b200/_build/, the shared library to
appt-spgemm-challenge_b200/libappt_spgemm.so. Sources are recompiled only when they (or a
header) are newer than their object.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
# A build variant (APPT_BUILD_VARIANT=<name>, with its own APPT_NVCC_DEFINES) goes to
# _build/<name>/ and _build/<name>/libappt_spgemm.so; load it with APPT_LIB=<that path>.
VARIANT = os.environ.get("APPT_BUILD_VARIANT", "")
BUILD = PKG / "_build" / VARIANT if VARIANT else PKG / "_build"
LIB = BUILD / "libappt_spgemm.so" if VARIANT else PKG / "libappt_spgemm.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=default",
          f"-I{INCLUDE}", f"-I{CSRC}"]
# Tuning constants (e.g. APPT_NVCC_DEFINES="APPT_RANK_MIN_BLOCKS=5") become -D flags.
COMMON += [f"-D{d}" for d in os.environ.get("APPT_NVCC_DEFINES", "").split() if d]


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, ptxas_info: bool) -> tuple[Path, str]:
    obj = BUILD / (src.name + ".o")
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if ptxas_info and src.suffix == ".cu":
        cmd[1:1] = ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    hdr = _headers_mtime()
    stamp = BUILD / "flags.txt"
    flags = " ".join(ARCH + COMMON)
    if not stamp.exists() or stamp.read_text() != flags:
        force = True
        stamp.write_text(flags)
    srcs = _sources()
    todo = []
    for s in srcs:
        obj = BUILD / (s.name + ".o")
        if force or ptxas_info or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, hdr):
            todo.append(s)
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose, ptxas_info), todo):
                logs.append((obj, log))
    objs = [BUILD / (s.name + ".o") for s in srcs]
    if force or todo or not LIB.exists():
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if ptxas_info:
        for obj, log in logs:
            print(f"== {obj.name}\n{log}")
    return LIB


DRIVER = BUILD / "spgemm_test"


def build_reference_driver(reference_dir, verbose: bool = False) -> Path | None:
    """Links the reference's own driver (src/main.cu of a reference checkout, compiled here
    unmodified) against libappt_spgemm.so in place of the reference's kernel objects and of
    src/matrix_utils.cu: the drop-in check of the library's reference-compatible exports. The
    executable is _build/spgemm_test (rpath to this directory). Returns None without the
    reference sources."""
    ref = Path(reference_dir)
    main_cu = ref / "src" / "main.cu"
    if not main_cu.exists():
        return None
    lib = build(verbose=verbose)
    if DRIVER.exists() and DRIVER.stat().st_mtime >= max(lib.stat().st_mtime,
                                                         main_cu.stat().st_mtime):
        return DRIVER
    cmd = [NVCC, *ARCH, "-O2", "-std=c++17", f"-I{ref / 'include'}", "-o", str(DRIVER),
           str(main_cu), f"-L{PKG}", "-lappt_spgemm", "-Xlinker", "-rpath", "-Xlinker",
           "$ORIGIN/..", "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"linking the reference driver failed:\n{r.stdout}\n{r.stderr}")
    return DRIVER


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    lib = build(a.force, a.verbose, a.ptxas_info)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
