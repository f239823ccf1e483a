"""Shared test setup: import paths, the `gpu` marker, and small helpers."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "appt-spgemm-challenge_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the engine")


# Value tolerance of the parity tests: |c - c_ref| <= 1e-12 * max(|c_ref|, sum_k |a_ik * b_kj|).
# The absolute-sum term bounds reordered fp64 summation with cancellation (values in U(-1,1)).
VALUE_RTOL = 1e-12


def abs_product(A, B=None, op="ab"):
    """|A| * |B| (same structure as the product), used as the per-entry error scale."""
    import oracle
    from appt_spgemm.matrices import Csr
    absA = Csr(A.rows, A.cols, A.row_ptr, A.col_idx, np.abs(A.val))
    absB = None if B is None else Csr(B.rows, B.cols, B.row_ptr, B.col_idx, np.abs(B.val))
    return oracle.spgemm(absA, absB, op=op)


def assert_same_structure(C, R):
    assert C.rows == R.rows, (C.rows, R.rows)
    rp_c = np.asarray(C.row_ptr, dtype=np.int64)
    rp_r = np.asarray(R.row_ptr, dtype=np.int64)
    assert np.array_equal(rp_c - rp_c[0], rp_r - rp_r[0]), "row_ptr differs"
    assert np.array_equal(np.asarray(C.col_idx), np.asarray(R.col_idx)), "col_idx differs"


def assert_values_close(C, R, scale, rtol=VALUE_RTOL):
    c = np.asarray(C.val)
    r = np.asarray(R.val)
    s = np.maximum(np.abs(r), np.asarray(scale.val))
    err = np.abs(c - r)
    bad = err > rtol * s + 1e-300
    assert not bad.any(), (f"{int(bad.sum())} values outside tolerance; worst rel "
                           f"{float((err / np.maximum(s, 1e-300)).max()):.3e}")


def gpu_available() -> bool:
    try:
        import appt_spgemm
        return appt_spgemm.device_count() > 0
    except Exception:
        return False


# ----------------------------------------------------------------------------- tier-forcing inputs
def _csr():
    from appt_spgemm.matrices import Csr
    return Csr


def tier_matrix_rows(n=1 << 18, seed=5):
    """Rows of very different lengths so that every symbolic and numeric tier is used."""
    Csr = _csr()
    rng = np.random.default_rng(seed)
    lens = np.minimum(rng.zipf(1.6, n), 700).astype(np.int64)
    lens[:4] = [600, 300, 150, 2000]
    lens[np.arange(4, n, 97)] = 0
    rows = []
    for i in range(n):
        L = int(lens[i])
        if L == 0:
            rows.append(np.zeros(0, np.int64))
            continue
        if i % 3 == 0:   # banded rows (dense tier candidates)
            c = np.unique(np.clip(i + rng.integers(-300, 300, L), 0, n - 1))
        else:
            c = np.unique(rng.integers(0, n, L))
        rows.append(c)
    rp = np.zeros(n + 1, np.int64)
    rp[1:] = np.cumsum([len(r) for r in rows])
    ci = np.concatenate(rows).astype(np.int32)
    return Csr(n, n, rp.astype(np.int32), ci, rng.uniform(-1, 1, ci.size))


def hub_matrix(n=1 << 17, hubs=24, hub_len=6000, seed=9):
    """Sparse rows plus a few hub rows with thousands of entries spread over the whole column
    range: rows of A*A that reach a hub have more than 4096 entries on a sparse, wide span (the
    CTA rank tier); the hub rows themselves span up to 2^17 columns."""
    Csr = _csr()
    rng = np.random.default_rng(seed)
    rows = []
    hub_ids = rng.choice(n, hubs, replace=False)
    for i in range(n):
        L = hub_len if i in hub_ids else int(rng.integers(1, 6))
        rows.append(np.unique(rng.integers(0, n, L)))
    rp = np.zeros(n + 1, np.int64)
    rp[1:] = np.cumsum([len(r) for r in rows])
    ci = np.concatenate(rows).astype(np.int32)
    return Csr(n, n, rp.astype(np.int32), ci, rng.uniform(-1, 1, ci.size))


def window_matrix(n=8192, seed=8):
    """Rows of A*A with more than ~600 entries packed into at most 16384 columns (the dense
    window tier)."""
    Csr = _csr()
    rng = np.random.default_rng(seed)
    rows = [np.unique(np.clip(i + rng.integers(-2000, 2000, 800), 0, n - 1)) for i in range(n)]
    rp = np.zeros(n + 1, np.int64)
    rp[1:] = np.cumsum([len(r) for r in rows])
    ci = np.concatenate(rows).astype(np.int32)
    return Csr(n, n, rp.astype(np.int32), ci, rng.uniform(-1, 1, ci.size))
