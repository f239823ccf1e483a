"""appt_spgemm_noalloc: the entry point for callers that cannot allocate during the multiply.

Some callers cannot call cudaMalloc while they multiply: a framework whose caching allocator owns
the whole device heap, code that runs where allocation is forbidden, or loops that size every
buffer once at start-up. For them the library computes C = A*B from device operands into device
buffers the caller owns and keeps its temporaries in one fixed device array inside the library.

These tests call it through the C ABI and check its C against the CPU oracle -- row_ptr and
col_idx bit for bit, values within the parity tolerance of the other GPU tests -- on consecutive
calls that reuse the shared array, including rows that take the CTA tiers, and compare it with the
regular entry point (appt_spgemm) on the same inputs. This file is collected last.
"""
import ctypes as ct

import numpy as np
import pytest

from conftest import (abs_product, assert_same_structure, assert_values_close, tier_matrix_rows,
                      window_matrix)

pytestmark = pytest.mark.gpu

import appt_spgemm as ap  # noqa: E402
import oracle  # noqa: E402
from appt_spgemm import matrices as M  # noqa: E402


def _bind():
    lib = ap.load()
    fn = lib.appt_spgemm_noalloc
    fn.argtypes = [ct.POINTER(ap.CsrIn), ct.POINTER(ap.CsrIn), ct.c_void_p, ct.c_void_p,
                   ct.c_void_p, ct.c_int64, ct.POINTER(ct.c_int64), ct.c_void_p]
    fn.restype = ct.c_int
    return fn


def _dev(torch, A, d):
    return (torch.from_numpy(np.ascontiguousarray(A.row_ptr, np.int32)).to(d),
            torch.from_numpy(np.ascontiguousarray(A.col_idx, np.int32)).to(d),
            torch.from_numpy(np.ascontiguousarray(A.val, np.float64)).to(d))


def _csr_in(A, t):
    return ap.CsrIn(A.rows, A.cols, A.nnz, t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr())


def _noalloc(torch, fn, A, B=None, capacity=None, device=0):
    """Runs the no-allocation entry on cuda:<device>; returns (status, nnz, C or None). Output
    buffers are pre-filled with garbage so that nothing unwritten can pass."""
    d = torch.device("cuda", device)
    with torch.cuda.device(d):
        tA = _dev(torch, A, d)
        tB = _dev(torch, B, d) if B is not None else None
        a = _csr_in(A, tA)
        b = _csr_in(B, tB) if B is not None else None
        cap = int(oracle.symbolic_counts(A, B).sum()) if capacity is None else capacity
        crp = torch.full((A.rows + 1,), -7, dtype=torch.int64, device=d)
        cci = torch.full((max(cap, 1),), -7, dtype=torch.int32, device=d)
        cva = torch.full((max(cap, 1),), np.nan, dtype=torch.float64, device=d)
        nnz = ct.c_int64(-1)
        stream = torch.cuda.current_stream(d)
        torch.cuda.synchronize(d)
        rc = fn(ct.byref(a), ct.byref(b) if b is not None else None, crp.data_ptr(),
                cci.data_ptr(), cva.data_ptr(), cap, ct.byref(nnz), stream.cuda_stream)
        torch.cuda.synchronize(d)
    cols = (B if B is not None else A).cols
    if rc != 0:
        return rc, nnz.value, M.Csr(A.rows, cols, crp.cpu().numpy(), None, None)
    n = nnz.value
    return rc, n, M.Csr(A.rows, cols, crp.cpu().numpy(), cci[:n].cpu().numpy(),
                        cva[:n].cpu().numpy())


def _check_against_oracle(C, A, B=None):
    R = oracle.spgemm(A, B)
    assert_same_structure(C, R)
    assert_values_close(C, R, abs_product(A, B))
    return R


def test_noalloc_matches_oracle_on_consecutive_calls():
    """Several calls in a row share the library's scratch array; each must match the oracle and
    the regular entry point. The tier matrix and the window matrix send rows to the CTA tiers
    (CTA hash, CTA rank, dense window), whose row counters live in that array too."""
    torch = pytest.importorskip("torch")
    fn = _bind()
    tier = tier_matrix_rows()
    win = window_matrix()
    cases = [(M.stencil27(g=20), None, ()),
             (tier, None, ("hash_block", "block_rank")),
             (M.random_csr(700, 700, 0.02, 3, empty_rows=0.1), None, ()),
             (win, None, ("window",)),
             (M.random_csr(300, 200, 0.03, 5), M.random_csr(200, 450, 0.03, 6), ()),
             (tier, None, ("hash_block", "block_rank")),
             (M.stencil27(g=20), None, ())]
    for A, B, cta_tiers in cases:
        rc, n, C = _noalloc(torch, fn, A, B)
        assert rc == 0, ap.last_error()
        R = _check_against_oracle(C, A, B)
        assert n == R.nnz
        Creg, st = ap.spgemm(A, B, return_stats=True)
        for t in cta_tiers:   # the classifier sent rows to this CTA tier
            assert st["tier_rows"][t] > 0, (t, st["tier_rows"])
        assert np.array_equal(C.col_idx, Creg.col_idx)


def test_noalloc_reports_size_when_capacity_is_short():
    torch = pytest.importorskip("torch")
    fn = _bind()
    A = M.stencil27(g=12)
    R = oracle.spgemm(A)
    rc, n, C = _noalloc(torch, fn, A, capacity=R.nnz - 1)
    assert rc == -5                       # APPT_ERR_TOO_LARGE
    assert n == R.nnz
    assert np.array_equal(C.row_ptr, R.row_ptr)
    rc, n, C = _noalloc(torch, fn, A)     # and a full-size retry succeeds
    assert rc == 0 and n == R.nnz
    _check_against_oracle(C, A)


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


def test_noalloc_rejects_sizes_beyond_int32():
    """Sizes the kernels would narrow to int32 are refused before anything runs."""
    torch = pytest.importorskip("torch")
    fn = _bind()
    d = torch.device("cuda:0")
    rp = torch.zeros(9, dtype=torch.int32, device=d)
    a = ap.CsrIn(8, 1 << 31, 0, rp.data_ptr(), 0, 0)
    b = ap.CsrIn(1 << 31, 8, 0, rp.data_ptr(), 0, 0)
    crp = torch.zeros(9, dtype=torch.int64, device=d)
    nnz = ct.c_int64(0)
    rc = fn(ct.byref(a), ct.byref(b), crp.data_ptr(), 0, 0, 0, ct.byref(nnz), None)
    assert rc == -1 and nnz.value == -1


def test_noalloc_on_a_second_device():
    """The scratch array and the kernels' shared-memory limits are per device: a call on cuda:1
    after calls on cuda:0 must work the same (skipped with one visible GPU)."""
    torch = pytest.importorskip("torch")
    if ap.device_count() < 2:
        pytest.skip("one visible GPU")
    fn = _bind()
    A = tier_matrix_rows(n=1 << 15)
    for dev in (0, 1, 0, 1):
        rc, n, C = _noalloc(torch, fn, A, device=dev)
        assert rc == 0, ap.last_error()
        _check_against_oracle(C, A)
