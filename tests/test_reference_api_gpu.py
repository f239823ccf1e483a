"""The reference-compatible entry points (include/spgemm.h names and layouts) through the C ABI."""
import ctypes as ct

import numpy as np
import pytest

from conftest import abs_product, assert_same_structure, assert_values_close

pytestmark = pytest.mark.gpu

import appt_spgemm as ap  # noqa: E402
import oracle  # noqa: E402
from appt_spgemm import matrices as M  # noqa: E402


@pytest.mark.parametrize("mempool", [False, True])
@pytest.mark.parametrize("name", sorted(ap.REFERENCE_ENTRIES))
def test_reference_entries(name, mempool):
    ap.set_mempool(mempool)
    op, att_quirk = ap.REFERENCE_ENTRIES[name]
    A = M.random_csr(240, 240 if op == "ab" else 97, 0.04, 21, empty_rows=0.1)
    C, cr, cc, cn = ap.reference_entry(name, A)
    R = oracle.spgemm(A, op=op)
    assert cn == R.nnz and cr == A.rows
    # att_* report C_cols = A_cols like the reference (spgemm_kernel_hash.cu:1103)
    assert cc == (A.cols if (op == "ab" or att_quirk) else A.rows)
    assert_same_structure(C, R)
    assert_values_close(C, R, abs_product(A, op=op))
    ap.set_mempool(False)


def _d2h(ptr, n, dtype):
    from cuda.bindings import runtime as rt
    out = np.zeros(n, dtype=dtype)
    if n:
        err, = rt.cudaMemcpy(out.ctypes.data, ptr, out.nbytes,
                             rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert int(err) == 0, err
    return out


def _cuda_free(ptr):
    from cuda.bindings import runtime as rt
    err, = rt.cudaFree(ptr)
    assert int(err) == 0, err


def test_build_csc_device_contract():
    torch = pytest.importorskip("torch")
    A = M.random_csr(300, 300, 0.03, 4)
    dev = torch.device("cuda:0")
    rp = torch.from_numpy(A.row_ptr).to(dev)
    ci = torch.from_numpy(A.col_idx).to(dev)
    va = torch.from_numpy(A.val).to(dev)
    torch.cuda.synchronize()
    cp, ri, vv = ct.c_void_p(), ct.c_void_p(), ct.c_void_p()
    ap.load().build_csc(rp.data_ptr(), ci.data_ptr(), va.data_ptr(), A.rows, A.nnz, ct.byref(cp),
                        ct.byref(ri), ct.byref(vv))
    assert cp.value and ri.value and vv.value, ap.last_error()
    R = oracle.transpose(A)
    assert np.array_equal(_d2h(cp.value, A.rows + 1, np.int32), R.row_ptr)
    assert np.array_equal(_d2h(ri.value, A.nnz, np.int32), R.col_idx)
    assert np.array_equal(_d2h(vv.value, A.nnz, np.float64), R.val)
    for p in (cp, ri, vv):
        _cuda_free(p.value)


def test_device_resident_row_block_upper():
    """A row block of A with B = A^T passed explicitly and op ab_upper/row_base reproduces the
    same rows of the full upper(A*A^T) -- the per-GPU shard of the multi-GPU A*A^T path."""
    torch = pytest.importorskip("torch")
    A = M.random_csr(400, 150, 0.05, 8)
    full = oracle.spgemm(A, op="aat_upper")
    T = oracle.transpose(A)
    dev = torch.device("cuda:0")
    rp = torch.from_numpy(A.row_ptr).to(dev)
    ci = torch.from_numpy(A.col_idx).to(dev)
    va = torch.from_numpy(A.val).to(dev)
    trp = torch.from_numpy(T.row_ptr).to(dev)
    tci = torch.from_numpy(T.col_idx).to(dev)
    tva = torch.from_numpy(T.val).to(dev)
    torch.cuda.synchronize()
    r0, r1 = 123, 301
    res = ap.spgemm_device(r1 - r0, A.cols, int(A.row_ptr[r1] - A.row_ptr[r0]),
                           rp.data_ptr() + 4 * r0, ci.data_ptr(), va.data_ptr(),
                           B=(T.rows, T.cols, T.nnz, trp.data_ptr(), tci.data_ptr(), tva.data_ptr()),
                           op="ab_upper", row_base=r0)
    crp = _d2h(res.row_ptr, res.rows + 1, np.int64)
    cci = _d2h(res.col_idx, res.nnz, np.int32)
    cva = _d2h(res.val, res.nnz, np.float64)
    res.free()
    lo, hi = int(full.row_ptr[r0]), int(full.row_ptr[r1])
    assert np.array_equal(crp, full.row_ptr[r0:r1 + 1] - lo)
    assert np.array_equal(cci, full.col_idx[lo:hi])
    assert np.allclose(cva, full.val[lo:hi], rtol=1e-12, atol=1e-14)
