"""appt_spgemm_noalloc: the entry point for callers that cannot allocate during the multiply.

It computes C = A*B from device operands into device buffers the caller owns, keeping its
temporaries in one fixed device array inside the library. These tests call it through the C ABI
and compare its C with the regular entry point's (appt_spgemm), with the tolerance the parity
tests use, on consecutive calls that reuse the shared array.
"""
import ctypes as ct

import numpy as np
import pytest

from conftest import VALUE_RTOL

pytestmark = pytest.mark.gpu

import appt_spgemm as ap  # noqa: E402
from appt_spgemm import matrices as M  # noqa: E402


def _bind():
    lib = ap.load()
    fn = lib.appt_spgemm_noalloc
    fn.argtypes = [ct.POINTER(ap.CsrIn), ct.POINTER(ap.CsrIn), ct.c_void_p, ct.c_void_p,
                   ct.c_void_p, ct.c_int64, ct.POINTER(ct.c_int64), ct.c_void_p]
    fn.restype = ct.c_int
    return fn


def _dev(torch, A):
    d = torch.device("cuda:0")
    return (torch.from_numpy(np.ascontiguousarray(A.row_ptr, np.int32)).to(d),
            torch.from_numpy(np.ascontiguousarray(A.col_idx, np.int32)).to(d),
            torch.from_numpy(np.ascontiguousarray(A.val, np.float64)).to(d))


def _csr_in(A, t):
    return ap.CsrIn(A.rows, A.cols, A.nnz, t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr())


def _noalloc(torch, fn, A, B=None, capacity=None):
    """Returns (status, nnz, C or None)."""
    tA = _dev(torch, A)
    tB = _dev(torch, B) if B is not None else None
    a = _csr_in(A, tA)
    b = _csr_in(B, tB) if B is not None else None
    ref_nnz = ap.spgemm(A, B).nnz if capacity is None else capacity
    d = torch.device("cuda:0")
    crp = torch.full((A.rows + 1,), -7, dtype=torch.int64, device=d)
    cci = torch.full((max(ref_nnz, 1),), -7, dtype=torch.int32, device=d)
    cva = torch.full((max(ref_nnz, 1),), np.nan, dtype=torch.float64, device=d)
    nnz = ct.c_int64(-1)
    stream = torch.cuda.current_stream(d)
    torch.cuda.synchronize()
    rc = fn(ct.byref(a), ct.byref(b) if b is not None else None, crp.data_ptr(), cci.data_ptr(),
            cva.data_ptr(), ref_nnz, ct.byref(nnz), stream.cuda_stream)
    torch.cuda.synchronize()
    if rc != 0:
        return rc, nnz.value, M.Csr(A.rows, (B or A).cols, crp.cpu().numpy(), None, None)
    n = nnz.value
    return rc, n, M.Csr(A.rows, (B or A).cols, crp.cpu().numpy(), cci[:n].cpu().numpy(),
                        cva[:n].cpu().numpy())


def _same(C, R):
    assert np.array_equal(C.row_ptr, R.row_ptr)
    assert np.array_equal(C.col_idx, R.col_idx)
    s = np.maximum(np.abs(R.val), 1e-300)
    assert np.all(np.abs(C.val - R.val) <= VALUE_RTOL * np.maximum(s, np.abs(C.val)))


def test_noalloc_matches_regular_entry_on_consecutive_calls():
    torch = pytest.importorskip("torch")
    fn = _bind()
    cases = [(M.stencil27(g=20), None),
             (M.random_csr(700, 700, 0.02, 3, empty_rows=0.1), None),
             (M.random_csr(300, 200, 0.03, 5), M.random_csr(200, 450, 0.03, 6)),
             (M.stencil27(g=20), None)]
    for A, B in cases:           # consecutive calls share the library's scratch array
        rc, n, C = _noalloc(torch, fn, A, B)
        assert rc == 0, ap.last_error()
        R = ap.spgemm(A, B)
        assert n == R.nnz
        _same(C, R)


def test_noalloc_reports_size_when_capacity_is_short():
    torch = pytest.importorskip("torch")
    fn = _bind()
    A = M.stencil27(g=12)
    R = ap.spgemm(A)
    rc, n, C = _noalloc(torch, fn, A, capacity=R.nnz - 1)
    assert rc == -5                       # APPT_ERR_TOO_LARGE
    assert n == R.nnz
    assert np.array_equal(C.row_ptr, R.row_ptr)
    rc, n, C = _noalloc(torch, fn, A)     # and a full-size retry succeeds
    assert rc == 0 and n == R.nnz
    _same(C, R)


def test_noalloc_rejects_rows_beyond_the_scratch_limit():
    torch = pytest.importorskip("torch")
    fn = _bind()
    rows = 3_000_000
    d = torch.device("cuda:0")
    rp = torch.zeros(rows + 1, dtype=torch.int32, device=d)
    a = ap.CsrIn(rows, rows, 0, rp.data_ptr(), 0, 0)
    crp = torch.zeros(rows + 1, dtype=torch.int64, device=d)
    nnz = ct.c_int64(0)
    rc = fn(ct.byref(a), None, crp.data_ptr(), 0, 0, 0, ct.byref(nnz), None)
    assert rc == -5
    assert "rows" in ap.last_error() and "64 MiB" in ap.last_error()
