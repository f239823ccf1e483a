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
