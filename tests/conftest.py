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


def abs_product(A, B=None, op="ab", row_base=0):
    """|A| * |B| (same structure as the product), used as the per-entry error scale."""
    import oracle
    from appt_spgemm.matrices import Csr
    absA = Csr(A.rows, A.cols, A.row_ptr, A.col_idx, np.abs(A.val))
    absB = None if B is None else Csr(B.rows, B.cols, B.row_ptr, B.col_idx, np.abs(B.val))
    return oracle.spgemm(absA, absB, op=op, row_base=row_base)


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


# ----------------------------------------------------------------------------- device helpers
class _CudaArray:
    """Zero-copy view of library-owned device memory for torch (__cuda_array_interface__)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def device_view(torch, ptr: int, n: int, dtype: str, device: int = 0):
    """torch tensor over n elements of type dtype ('i4', 'i8', 'f8') at device address ptr."""
    if n == 0:
        return torch.zeros(0, dtype={"i4": torch.int32, "i8": torch.int64,
                                     "f8": torch.float64}[dtype], device=f"cuda:{device}")
    return torch.as_tensor(_CudaArray(ptr, n, "<" + dtype), device=f"cuda:{device}")


def to_device(torch, A, device: int = 0):
    """A's three arrays as device tensors (int32, int32, float64)."""
    d = torch.device("cuda", device)
    return (torch.from_numpy(np.ascontiguousarray(A.row_ptr, np.int32)).to(d),
            torch.from_numpy(np.ascontiguousarray(A.col_idx, np.int32)).to(d),
            torch.from_numpy(np.ascontiguousarray(A.val, np.float64)).to(d))


def select_rows(A, rows):
    """CSR of the listed rows of A (in the given order)."""
    from appt_spgemm.matrices import Csr
    rows = np.asarray(rows, np.int64)
    rp = np.asarray(A.row_ptr, np.int64)
    lens = rp[rows + 1] - rp[rows]
    out_rp = np.zeros(rows.size + 1, np.int64)
    np.cumsum(lens, out=out_rp[1:])
    idx = segment_index(rp[rows], lens)
    return Csr(int(rows.size), A.cols, out_rp.astype(np.int32), np.asarray(A.col_idx)[idx],
               np.asarray(A.val)[idx])


def segment_index(starts, lens):
    """Concatenation of arange(s, s + l) for every (s, l) pair (int64)."""
    starts = np.asarray(starts, np.int64)
    lens = np.asarray(lens, np.int64)
    total = int(lens.sum())
    if total == 0:
        return np.zeros(0, np.int64)
    off = np.zeros(lens.size, np.int64)
    np.cumsum(lens[:-1], out=off[1:])
    return np.repeat(starts - off, lens) + np.arange(total, dtype=np.int64)
