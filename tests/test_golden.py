"""Pins the CPU oracle (and, on a GPU, the engine) to outputs of the reference's own CUDA build.

Fixtures in tests/golden/ were produced by tests/golden/make_golden.py running
oracle/_ref/ref_spgemm (unmodified reference sources, sm_100a) on one B200. Inputs are
regenerated here from the same seeds. Structure must match bit for bit; values within the
parity tolerance (the reference sums in a different order: atomics / warp reductions).
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import VALUE_RTOL

import oracle
from appt_spgemm import matrices as M

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = GOLDEN / "manifest.json"

OPS = {"adaptive": "ab", "hash": "ab", "merge3": "ab", "manual": "ab",
       "att_adaptive": "aat_upper", "att_hash": "aat_upper", "att_merge3": "aat_upper"}


def _cases(kind):
    if not MANIFEST.exists():
        return []
    man = json.loads(MANIFEST.read_text())
    out = []
    for key, ent in sorted(man.items()):
        if ent.get("file") and ent["file"].endswith(kind):
            out.append(pytest.param(key, ent, id=key))
    return out


_INPUTS = {}


def _input(ent):
    k = (ent["generator"], json.dumps(ent["kwargs"], sort_keys=True))
    if k not in _INPUTS:
        _INPUTS[k] = getattr(M, ent["generator"])(**ent["kwargs"])
    return _INPUTS[k]


def _scale(A, op):
    absA = M.Csr(A.rows, A.cols, A.row_ptr, A.col_idx, np.abs(A.val))
    return oracle.spgemm(absA, op=op)


def check_full(C, fx, scale):
    assert np.array_equal(np.asarray(C.row_ptr, np.int64), fx["row_ptr"].astype(np.int64))
    assert np.array_equal(np.asarray(C.col_idx), fx["col_idx"])
    s = np.maximum(np.abs(fx["val"]), scale.val)
    assert np.all(np.abs(np.asarray(C.val) - fx["val"]) <= VALUE_RTOL * s + 1e-300)


def check_digest(C, d, scale):
    assert C.nnz == d["nnz"]
    assert hashlib.sha256(np.asarray(C.row_ptr).astype("<i4").tobytes()).hexdigest() == \
        d["row_ptr_sha256"]
    assert hashlib.sha256(np.asarray(C.col_idx).astype("<i4").tobytes()).hexdigest() == \
        d["col_idx_sha256"]
    rp = np.asarray(C.row_ptr, np.int64)
    for i, row in d["sample_rows"].items():
        i = int(i)
        lo, hi = rp[i], rp[i + 1]
        assert np.asarray(C.col_idx[lo:hi]).tolist() == row["cols"]
        ref = np.asarray(row["vals"])
        s = np.maximum(np.abs(ref), scale.val[lo:hi])
        assert np.all(np.abs(np.asarray(C.val[lo:hi]) - ref) <= VALUE_RTOL * s + 1e-300)
    assert abs(float(np.sum(np.abs(C.val))) - d["val_abs_sum"]) <= 1e-9 * d["val_abs_sum"]


def test_fixtures_present():
    assert MANIFEST.exists(), "golden fixtures missing: run tests/golden/make_golden.py on a GPU"
    man = json.loads(MANIFEST.read_text())
    assert any(e.get("file") for e in man.values())


@pytest.mark.parametrize("key,ent", _cases(".npz"))
def test_oracle_matches_reference_small(key, ent):
    A = _input(ent)
    op = OPS[ent["method"]]
    fx = np.load(GOLDEN / ent["file"])
    C = oracle.spgemm(A, op=op)
    check_full(C, fx, _scale(A, op))


@pytest.mark.parametrize("key,ent", _cases(".json"))
def test_oracle_matches_reference_digest(key, ent):
    A = _input(ent)
    op = OPS[ent["method"]]
    d = json.loads((GOLDEN / ent["file"]).read_text())
    C = oracle.spgemm(A, op=op)
    check_digest(C, d, _scale(A, op))


@pytest.mark.gpu
@pytest.mark.parametrize("key,ent", _cases(".npz") + _cases(".json"))
def test_engine_matches_reference(key, ent):
    import appt_spgemm as ap
    A = _input(ent)
    op = OPS[ent["method"]]
    method = {"adaptive": "adaptive", "hash": "hash", "merge3": "merge", "manual": "esc",
              "att_adaptive": "adaptive", "att_hash": "hash", "att_merge3": "merge"}[ent["method"]]
    C = ap.spgemm(A, op=op, method=method)
    if ent["file"].endswith(".npz"):
        check_full(C, np.load(GOLDEN / ent["file"]), _scale(A, op))
    else:
        check_digest(C, json.loads((GOLDEN / ent["file"]).read_text()), _scale(A, op))


# ----------------------------------------------------------------------------- estimator pins
ESTIMATES = GOLDEN / "estimates.json"


def _est_cases():
    if not ESTIMATES.exists():
        return []
    est = json.loads(ESTIMATES.read_text())
    return [pytest.param(k, e, id=k) for k, e in sorted(est.items())]


@pytest.mark.parametrize("key,ent", _est_cases())
def test_oracle_estimate_matches_reference_total(key, ent):
    """The oracle's restatement of the reference's MinHash and HyperLogLog sizing estimates sums
    to the reference's own "[hash] total_est" (src/spgemm_kernel_hash.cu:925), recorded by
    tests/golden/make_golden.py --estimates from the reference's CUDA build."""
    A = _input(ent)
    att = ent["method"].startswith("att")
    mh = oracle.estimate_row_nnz(A, att=att, estimator="minhash").astype(np.int64)
    hll = oracle.estimate_row_nnz(A, att=att, estimator="hll").astype(np.int64)
    assert int(mh.sum()) == ent["total_est"]
    assert int(hll.sum()) == ent["total_est_hll"]


@pytest.mark.gpu
@pytest.mark.parametrize("key,ent", _est_cases())
def test_engine_estimate_matches_reference_total(key, ent):
    """The engine's estimator (appt_estimate_row_nnz) sums to the reference's total_est and
    agrees row by row with the oracle's restatement."""
    import appt_spgemm as ap
    A = _input(ent)
    att = ent["method"].startswith("att")
    for name, key_total in (("minhash", "total_est"), ("hll", "total_est_hll")):
        e = ap.estimate_row_nnz(A, att=att, estimator=name).astype(np.int64)
        assert int(e.sum()) == ent[key_total], name
        r = oracle.estimate_row_nnz(A, att=att, estimator=name).astype(np.int64)
        assert np.array_equal(e, r), (name, int((e != r).sum()))
