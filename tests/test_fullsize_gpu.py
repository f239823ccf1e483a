"""Full-size parity of the large workloads, which the other GPU tests only cover in miniature.

* banded n = 2^22 (16 entries per row within +-256 of the diagonal, C = A*A, 1.07e9 products,
  C of 9.2e8 entries): every entry of C against the CPU oracle, row block by row block.
* R-MAT 2^20 (16M edges, C = A*A, 2.09e10 products, C of 9.7e9 entries -- 117 GB, kept on the
  device): for every row, the exact entry count and the exact sum of column ids against the
  oracle's symbolic pass, and the row's value sum against A (B 1) (linearity); then the rows
  above the 99.9th percentile of products plus 10,000 seeded random rows entry by entry.
* Zipf 2^18 x 2^16, C = A*A^T (3.98e11 products, C of about 825 GB, formed in row blocks against
  a device-built A^T): the first, a middle and the last row block with the same per-row
  invariants and 200 sampled rows each, and one block of the upper-triangle variant.

Structure is compared bit for bit; values within |c - r| <= 1e-12 max(|r|, sum |a b|) per entry,
and per-row value sums within 2 (products + 1) eps sum |a| |b| (both sums reorder up to that many
roundings).
"""
import numpy as np
import pytest

from conftest import (abs_product, assert_same_structure, assert_values_close, device_view,
                      segment_index, select_rows, to_device)

pytestmark = pytest.mark.gpu

import appt_spgemm as ap  # noqa: E402
import oracle  # noqa: E402
from appt_spgemm import matrices as M  # noqa: E402
from appt_spgemm.streaming import cut_blocks, row_products_aat  # noqa: E402

EPS = np.finfo(np.float64).eps


def _torch():
    return pytest.importorskip("torch")


def _run(torch, A, tA, B=None, tB=None, op="ab", r0=0, r1=None):
    """Engine call on rows [r0, r1) of device A (B = A when None); C stays on the device."""
    r1 = A.rows if r1 is None else r1
    rp = np.asarray(A.row_ptr, np.int64)
    bspec = None
    if B is not None:
        bspec = (B.rows, B.cols, B.nnz, tB[0].data_ptr(), tB[1].data_ptr(), tB[2].data_ptr())
    elif r1 - r0 != A.rows:
        bspec = (A.rows, A.cols, A.nnz, tA[0].data_ptr(), tA[1].data_ptr(), tA[2].data_ptr())
    return ap.spgemm_device(r1 - r0, A.cols, int(rp[r1] - rp[r0]), tA[0].data_ptr() + 4 * r0,
                            tA[1].data_ptr(), tA[2].data_ptr(), B=bspec, op=op, row_base=r0)


def _views(torch, res):
    rp = device_view(torch, res.row_ptr, res.rows + 1, "i8")
    ci = device_view(torch, res.col_idx, res.nnz, "i4")
    va = device_view(torch, res.val, res.nnz, "f8")
    return rp.cpu().numpy(), ci, va


def _row_sums_device(torch, rp_h, ci, va, max_entries=1 << 27):
    """Per-row sums of column ids (exact, int64) and of values of a device CSR, in chunks."""
    rows = rp_h.size - 1
    csum = np.zeros(rows, np.int64)
    vsum = np.zeros(rows, np.float64)
    r0 = 0
    while r0 < rows:
        r1 = int(np.searchsorted(rp_h, rp_h[r0] + max_entries, side="right")) - 1
        r1 = min(max(r1, r0 + 1), rows)
        e0, e1 = int(rp_h[r0]), int(rp_h[r1])
        lens = torch.from_numpy(np.diff(rp_h[r0:r1 + 1])).to(ci.device)
        rid = torch.repeat_interleave(torch.arange(r1 - r0, device=ci.device), lens,
                                      output_size=e1 - e0)
        cs = torch.zeros(r1 - r0, dtype=torch.int64, device=ci.device)
        cs.index_add_(0, rid, ci[e0:e1].to(torch.int64))
        vs = torch.zeros(r1 - r0, dtype=torch.float64, device=ci.device)
        vs.index_add_(0, rid, va[e0:e1])
        csum[r0:r1] = cs.cpu().numpy()
        vsum[r0:r1] = vs.cpu().numpy()
        r0 = r1
    return csum, vsum


def _gather_rows(torch, rp_h, ci, va, rows, cols):
    """Host CSR of the listed rows of a device CSR."""
    rows = np.asarray(rows, np.int64)
    lens = rp_h[rows + 1] - rp_h[rows]
    out_rp = np.zeros(rows.size + 1, np.int64)
    np.cumsum(lens, out=out_rp[1:])
    idx = torch.from_numpy(segment_index(rp_h[rows], lens)).to(ci.device)
    return M.Csr(int(rows.size), cols, out_rp, ci[idx].cpu().numpy(), va[idx].cpu().numpy())


def _check_invariants(torch, res, A, B, products):
    """Every row: entry count and column-id sum exact, value sum within its rounding bound."""
    rp_h, ci, va = _views(torch, res)
    nnz_o, csum_o = oracle.symbolic_sums(A, B)
    assert np.array_equal(np.diff(rp_h), nnz_o), "row entry counts differ from the oracle"
    csum, vsum = _row_sums_device(torch, rp_h, ci, va)
    assert np.array_equal(csum, csum_o), "row column-id sums differ from the oracle"
    s, sa = oracle.row_value_sums(A, B)
    bad = np.abs(vsum - s) > 2.0 * (products + 1) * EPS * sa + 1e-300
    assert not bad.any(), f"{int(bad.sum())} row value sums outside their rounding bound"
    return rp_h, ci, va


def _check_rows(torch, rp_h, ci, va, A, B, rows, cols):
    sub = select_rows(A, rows)
    C = _gather_rows(torch, rp_h, ci, va, rows, cols)
    R = oracle.spgemm(sub, B)
    assert_same_structure(C, R)
    assert_values_close(C, R, abs_product(sub, B))


def test_banded_2e22_every_entry():
    torch = _torch()
    A = M.banded()
    tA = to_device(torch, A)
    res = _run(torch, A, tA)
    try:
        assert res.stats["products"] == int(oracle.row_products(A).sum())
        rp_h, ci, va = _views(torch, res)
        step = 1 << 20
        for r0 in range(0, A.rows, step):
            r1 = min(r0 + step, A.rows)
            blk = select_rows(A, np.arange(r0, r1))
            C = _gather_rows(torch, rp_h, ci, va, np.arange(r0, r1), A.cols)
            R = oracle.spgemm(blk, A)
            assert_same_structure(C, R)
            assert_values_close(C, R, abs_product(blk, A))
    finally:
        res.free()
        ap.release_cached()


def test_rmat_2e20_invariants_and_sampled_rows():
    torch = _torch()
    A = M.rmat()
    P = oracle.row_products(A)
    tA = to_device(torch, A)
    res = _run(torch, A, tA)
    try:
        assert res.stats["products"] == int(P.sum())
        assert res.nnz > (1 << 32)   # C needs int64 offsets
        rp_h, ci, va = _check_invariants(torch, res, A, A, P)
        heavy = np.nonzero(P > np.percentile(P, 99.9))[0]
        rnd = np.random.default_rng(20).choice(A.rows, 10000, replace=False)
        sample = np.unique(np.concatenate([heavy, rnd]))
        _check_rows(torch, rp_h, ci, va, A, A, sample, A.cols)
    finally:
        res.free()
        ap.release_cached()


def test_zipf_att_row_blocks():
    torch = _torch()
    A = M.zipf_att()
    tA = to_device(torch, A)
    d = tA[0].device
    t_rp = torch.empty(A.cols + 1, dtype=torch.int32, device=d)
    t_ci = torch.empty(A.nnz, dtype=torch.int32, device=d)
    t_va = torch.empty(A.nnz, dtype=torch.float64, device=d)
    ap.transpose_into_device(A.rows, A.cols, A.nnz, tA[0].data_ptr(), tA[1].data_ptr(),
                             tA[2].data_ptr(), t_rp.data_ptr(), t_ci.data_ptr(), t_va.data_ptr())
    AT = M.Csr(A.cols, A.rows, t_rp.cpu().numpy(), t_ci.cpu().numpy(), t_va.cpu().numpy())
    R_T = oracle.transpose(A)
    assert np.array_equal(AT.row_ptr, R_T.row_ptr) and np.array_equal(AT.col_idx, R_T.col_idx)
    assert np.array_equal(AT.val, R_T.val)
    tAT = (t_rp, t_ci, t_va)
    prods = row_products_aat(A)
    bounds = cut_blocks(prods, 1 << 32)
    nb = len(bounds) - 1
    assert nb > 10
    rng = np.random.default_rng(21)
    try:
        for b in (0, nb // 2, nb - 1):
            r0, r1 = bounds[b], bounds[b + 1]
            blk = select_rows(A, np.arange(r0, r1))
            res = _run(torch, A, tA, AT, tAT, "ab", r0, r1)
            try:
                assert res.stats["products"] == int(prods[r0:r1].sum())
                rp_h, ci, va = _check_invariants(torch, res, blk, AT, prods[r0:r1])
                rows = np.sort(rng.choice(r1 - r0, min(200, r1 - r0), replace=False))
                _check_rows(torch, rp_h, ci, va, blk, AT, rows, A.rows)
            finally:
                res.free()
        # the upper-triangle variant (the reference's att entries) on a middle block
        r0, r1 = bounds[nb // 2], bounds[nb // 2 + 1]
        blk = select_rows(A, np.arange(r0, r1))
        res = _run(torch, A, tA, AT, tAT, "ab_upper", r0, r1)
        try:
            rp_h, ci, va = _views(torch, res)
            nnz_o, csum_o = oracle.symbolic_sums(blk, AT, upper=True, row_base=r0)
            assert np.array_equal(np.diff(rp_h), nnz_o)
            csum, _ = _row_sums_device(torch, rp_h, ci, va)
            assert np.array_equal(csum, csum_o)
            q0 = (r1 - r0) // 2
            q1 = min(q0 + 100, r1 - r0)
            sub = select_rows(blk, np.arange(q0, q1))
            C = _gather_rows(torch, rp_h, ci, va, np.arange(q0, q1), A.rows)
            R = oracle.spgemm(sub, AT, op="ab_upper", row_base=r0 + q0)
            assert_same_structure(C, R)
            assert_values_close(C, R, abs_product(sub, AT, op="ab_upper", row_base=r0 + q0))
        finally:
            res.free()
    finally:
        ap.release_cached()
