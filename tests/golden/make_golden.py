"""Generate golden fixtures from the reference's own CUDA build.

Runs oracle/_ref/ref_spgemm (the unmodified reference sources compiled for sm_100a by
oracle/Makefile) on seeded inputs from appt_spgemm.matrices and stores its outputs:

  * small cases: full C (row_ptr, col_idx, val) as compressed .npz;
  * workload-size cases: sha256 digests of row_ptr / col_idx plus value checksums and the full
    contents of 64 sampled rows (.json).

Needs a GPU (the reference is CUDA-only). Usage, from the repository root:

  python tests/golden/make_golden.py --out gpurun_out/golden

then copy the files into tests/golden/. The inputs are regenerated from the same seeds by the
tests, so only the reference's outputs are stored.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "appt-spgemm-challenge_b200"))
from appt_spgemm import matrices as M  # noqa: E402

REF = ROOT / "oracle" / "_ref" / "ref_spgemm"
FULL_MAX_NNZ = 20000   # larger outputs are stored as digests

# name -> (generator kwargs, reference methods). The att_* methods run on square inputs only:
# for A_cols < A_rows the reference's att paths size B by A_rows and bucket by A_cols
# (src/spgemm_kernel_formulations.cu:73-81, src/spgemm_merge.cu:692-694).
SMALL = {
    "uniform8_n512": ("uniform8", {"n": 512}, ["adaptive", "hash", "merge3", "manual"]),
    "stencil27_g12": ("stencil27", {"g": 12}, ["adaptive", "hash", "merge3", "manual"]),
    "random_300_empty": ("random_csr", {"rows": 300, "cols": 300, "density": 0.04, "seed": 21,
                                         "empty_rows": 0.1},
                         ["adaptive", "hash", "merge3", "manual", "att_adaptive", "att_hash",
                          "att_merge3"]),
    "banded_n4096": ("banded", {"n": 4096}, ["adaptive", "hash", "merge3"]),
    "rmat_s10": ("rmat", {"scale": 10}, ["adaptive", "hash", "merge3", "att_adaptive"]),
}
LARGE = {
    "uniform8_n4096": ("uniform8", {}, ["adaptive", "merge3", "hash"]),
    "stencil27_g64": ("stencil27", {}, ["adaptive", "hash"]),
    "stencil27_g24": ("stencil27", {"g": 24}, ["adaptive", "hash", "att_adaptive"]),
}


def gen(name: str, kw: dict) -> M.Csr:
    return getattr(M, name)(**kw)


def run_ref(method: str, A: M.Csr, td: Path):
    inp = td / "in.bin"
    out = td / "out.bin"
    M.save_bin(inp, A)
    if out.exists():
        out.unlink()
    r = subprocess.run([str(REF), method, str(inp), "--out", str(out), "--warmup", "0",
                        "--repeat", "1"], capture_output=True, text=True, timeout=900)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{\"products\"")]
    info = json.loads(lines[-1]) if lines else {"error": r.stderr.strip().splitlines()[-3:]}
    if r.returncode != 0 or not out.exists():
        return None, info
    return M.load_bin(out), info


def digest(C: M.Csr, rng) -> dict:
    """sha256 of the structure, value sums, and the full contents of up to 24 of 64 randomly
    chosen rows (rows longer than 512 entries are skipped to keep the fixture small)."""
    rows = np.sort(rng.choice(C.rows, size=min(64, C.rows), replace=False))
    rp = C.row_ptr.astype(np.int64)
    rows = [i for i in rows if rp[i + 1] - rp[i] <= 512][:24]
    sample = {int(i): {"cols": C.col_idx[rp[i]:rp[i + 1]].tolist(),
                       "vals": C.val[rp[i]:rp[i + 1]].tolist()} for i in rows}
    return {"rows": C.rows, "nnz": C.nnz,
            "row_ptr_sha256": hashlib.sha256(C.row_ptr.astype("<i4").tobytes()).hexdigest(),
            "col_idx_sha256": hashlib.sha256(C.col_idx.astype("<i4").tobytes()).hexdigest(),
            "val_sum": float(np.sum(C.val)), "val_abs_sum": float(np.sum(np.abs(C.val))),
            "sample_rows": sample}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="gpurun_out/golden")
    a = ap.parse_args()
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    manifest = {}
    with tempfile.TemporaryDirectory() as tdn:
        td = Path(tdn)
        for case, (g, kw, methods) in SMALL.items():
            A = gen(g, kw)
            for meth in methods:
                C, info = run_ref(meth, A, td)
                key = f"{case}__{meth}"
                manifest[key] = {"generator": g, "kwargs": kw, "method": meth, "info": info,
                                 "file": None}
                if C is not None and C.nnz <= FULL_MAX_NNZ:
                    f = f"{key}.npz"
                    np.savez_compressed(out / f, row_ptr=C.row_ptr, col_idx=C.col_idx, val=C.val,
                                        rows=C.rows, cols=C.cols)
                    manifest[key]["file"] = f
                elif C is not None:
                    f = f"{key}.json"
                    (out / f).write_text(json.dumps(digest(C, np.random.default_rng(0))))
                    manifest[key]["file"] = f
                print(key, info, flush=True)
        for case, (g, kw, methods) in LARGE.items():
            A = gen(g, kw)
            for meth in methods:
                C, info = run_ref(meth, A, td)
                key = f"{case}__{meth}"
                manifest[key] = {"generator": g, "kwargs": kw, "method": meth, "info": info,
                                 "file": None}
                if C is not None:
                    f = f"{key}.json"
                    (out / f).write_text(json.dumps(digest(C, np.random.default_rng(0))))
                    manifest[key]["file"] = f
                print(key, info, flush=True)
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
