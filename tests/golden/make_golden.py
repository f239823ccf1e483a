"""Generate golden fixtures from the reference's own CUDA build.

Runs oracle/_ref/ref_spgemm (the unmodified reference sources compiled for sm_100a by
oracle/Makefile) on seeded inputs from appt_spgemm.matrices and stores its outputs:

  * small cases: full C (row_ptr, col_idx, val) as compressed .npz;
  * workload-size cases: sha256 digests of row_ptr / col_idx plus value checksums and the full
    contents of 64 sampled rows (.json).

Every run of the reference's hash path also prints the sum of its per-row output estimates
("[hash] total_est=<n>" on stderr, src/spgemm_kernel_hash.cu:925); it is kept in each case's
manifest entry (info.total_est). With --estimates the script instead runs the ESTIMATES cases --
inputs with at least 100000 nonzeros, where the reference sizes rows by its MinHash (default) or
HyperLogLog (EST_METHOD=hll) estimate rather than by exact products -- and writes only
estimates.json with both sums per case.

Needs a GPU (the reference is CUDA-only). Usage, from the repository root:

  python tests/golden/make_golden.py [--out DIR] [--estimates]

DIR defaults to tests/golden. The inputs are regenerated from the same seeds by the tests, so
only the reference's outputs are stored.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
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
# Estimator pins: (generator, kwargs, reference method). All have >= 100000 nonzeros, and on
# each the oracle's restatement of both estimators never sizes a row below its exact nnz (the
# reference writes a row's entries at its estimate-sized slot, so an underestimate would spill
# into the next row's slot; R-MAT inputs do underestimate some rows and are left out).
ESTIMATES = {
    "stencil27_g24": ("stencil27", {"g": 24}, "hash"),
    "stencil27_g40": ("stencil27", {"g": 40}, "hash"),
    "stencil27_g64": ("stencil27", {}, "hash"),
    "uniform8_n32768": ("uniform8", {"n": 32768}, "hash"),
    "banded_n32768": ("banded", {"n": 32768}, "hash"),
    "random_3000": ("random_csr", {"rows": 3000, "cols": 3000, "density": 0.02, "seed": 31},
                    "hash"),
    "stencil27_g24_att": ("stencil27", {"g": 24}, "att_hash"),
}
LARGE = {
    "uniform8_n4096": ("uniform8", {}, ["adaptive", "merge3", "hash"]),
    "stencil27_g64": ("stencil27", {}, ["adaptive", "hash"]),
    "stencil27_g24": ("stencil27", {"g": 24}, ["adaptive", "hash", "att_adaptive"]),
}


def gen(name: str, kw: dict) -> M.Csr:
    return getattr(M, name)(**kw)


def total_est(stderr: str):
    """The last "[hash] total_est=<n>" the reference printed, or None."""
    m = re.findall(r"\[hash\] total_est=(-?\d+)", stderr)
    return int(m[-1]) if m else None


def run_ref(method: str, A: M.Csr, td: Path, est_method: str | None = None):
    inp = td / "in.bin"
    out = td / "out.bin"
    M.save_bin(inp, A)
    if out.exists():
        out.unlink()
    env = dict(os.environ)
    env.pop("EST_METHOD", None)
    if est_method:
        env["EST_METHOD"] = est_method
    r = subprocess.run([str(REF), method, str(inp), "--out", str(out), "--warmup", "0",
                        "--repeat", "1"], capture_output=True, text=True, timeout=900, env=env)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{\"products\"")]
    info = json.loads(lines[-1]) if lines else {"error": r.stderr.strip().splitlines()[-3:]}
    te = total_est(r.stderr)
    if te is not None:
        info["total_est"] = te
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
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden"))
    ap.add_argument("--estimates", action="store_true",
                    help="only the estimator pins (writes estimates.json)")
    a = ap.parse_args()
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    if a.estimates:
        est = {}
        with tempfile.TemporaryDirectory() as tdn:
            td = Path(tdn)
            for case, (g, kw, meth) in ESTIMATES.items():
                A = gen(g, kw)
                _, info = run_ref(meth, A, td)
                _, info_hll = run_ref(meth, A, td, est_method="hll")
                est[case] = {"generator": g, "kwargs": kw, "method": meth, "nnz_a": A.nnz,
                             "total_est": info.get("total_est"),
                             "total_est_hll": info_hll.get("total_est"),
                             "c_nnz": info.get("c_nnz"), "products": info.get("products")}
                print(case, est[case], flush=True)
        (out / "estimates.json").write_text(json.dumps(est, indent=1))
        return 0
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
