"""Parity of the CUDA engine (through the C ABI) with the CPU oracle.

Structure (row_ptr, col_idx) must be bit-exact; values within
|c - c_ref| <= 1e-12 * max(|c_ref|, sum_k |a_ik b_kj|) (conftest.VALUE_RTOL).
"""
import numpy as np
import pytest

from conftest import (abs_product, assert_same_structure, assert_values_close, hub_matrix,
                      tier_matrix_rows, window_matrix)

pytestmark = pytest.mark.gpu

import appt_spgemm as ap  # noqa: E402
import oracle  # noqa: E402
from appt_spgemm import matrices as M  # noqa: E402

METHODS = ["adaptive", "hash", "merge", "esc"]


def check(A, B=None, op="ab", method="adaptive"):
    C, st = ap.spgemm(A, B, op=op, method=method, return_stats=True)
    R = oracle.spgemm(A, B, op=op)
    assert_same_structure(C, R)
    assert_values_close(C, R, abs_product(A, B, op))
    assert st["c_nnz"] == R.nnz
    return C, st


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_square(method, seed):
    A = M.random_csr(300, 300, 0.03 + 0.02 * seed, seed, empty_rows=0.1)
    check(A, method=method)


@pytest.mark.parametrize("op", ["ab", "aat_upper"])
@pytest.mark.parametrize("name", ["uniform8", "stencil27", "rmat", "banded"])
def test_small_problem_path_and_general_pipeline_agree(name, op, monkeypatch):
    """Small inputs take the unbinned small-problem path; the general binned pipeline
    (APPT_NO_SMALL_PATH=1) must give the same C bit for bit where both use the sequential
    rank tier, and both match the oracle."""
    A = M.make(name, small=True)
    C1, st1 = check(A, op=op)
    monkeypatch.setenv("APPT_NO_SMALL_PATH", "1")
    C2, st2 = check(A, op=op)
    assert np.array_equal(C1.col_idx, C2.col_idx)
    rank1 = sum(st1["tier_rows"][t] for t in ("rank2k", "rank4k", "rank8k"))
    if st2["tier_rows"]["hash_block"] == st2["tier_rows"]["window"] == \
            st2["tier_rows"]["block_rank"] == 0 and rank1 == A.rows:
        assert np.array_equal(C1.val, C2.val)


def _with_wide_rows(A, rows, per_row, seed):
    """A copy of A whose given rows are replaced by `per_row` columns spread over all columns."""
    rng = np.random.default_rng(seed)
    rp = np.asarray(A.row_ptr, np.int64)
    cols = [A.col_idx[rp[i]:rp[i + 1]] for i in range(A.rows)]
    vals = [A.val[rp[i]:rp[i + 1]] for i in range(A.rows)]
    for i in rows:
        cols[i] = np.unique(rng.integers(0, A.cols, per_row)).astype(np.int32)
        vals[i] = rng.uniform(-1, 1, cols[i].size)
    nrp = np.zeros(A.rows + 1, np.int64)
    nrp[1:] = np.cumsum([c.size for c in cols])
    return M.Csr(A.rows, A.cols, nrp.astype(np.int32), np.concatenate(cols),
                 np.concatenate(vals))


@pytest.mark.parametrize("case", ["every_row_wide", "few_rows_wide"])
def test_small_path_fallback_equals_general_pipeline(case, monkeypatch):
    """A's rows are within the small-problem path's limit (2^17), but rows of C are too wide for
    it: every row (uniform columns over 2^17) or the rows near a few planted wide rows of a
    banded matrix. The path stops early and hands the call to the binned pipeline, whose result
    must equal a call that skips the small path outright, bit for bit, and the oracle."""
    n = 1 << 17
    if case == "every_row_wide":
        A = M.uniform8(n)
    else:
        A = _with_wide_rows(M.banded(n, per_row=8, half_width=64, seed=6), [5, 70000, 131000],
                            8, seed=7)
    C1, st1 = check(A)
    monkeypatch.setenv("APPT_NO_SMALL_PATH", "1")
    C2, st2 = check(A)
    assert np.array_equal(C1.row_ptr, C2.row_ptr)
    assert np.array_equal(C1.col_idx, C2.col_idx)
    assert np.array_equal(C1.val, C2.val)
    assert st1["tier_rows"] == st2["tier_rows"]


@pytest.mark.parametrize("method", METHODS)
@pytest.mark.parametrize("op", ["aat", "aat_upper"])
def test_random_aat(method, op):
    A = M.random_csr(257, 131, 0.05, 7, empty_rows=0.05)
    check(A, op=op, method=method)


@pytest.mark.parametrize("method", METHODS)
def test_rectangular_ab(method):
    A = M.random_csr(200, 150, 0.04, 11)
    B = M.random_csr(150, 333, 0.03, 12)
    check(A, B, method=method)


@pytest.mark.parametrize("name", list(M.WORKLOADS))
@pytest.mark.parametrize("method", METHODS)
def test_workload_families_small(name, method):
    A = M.make(name, small=True)
    op = M.WORKLOADS[name][1]
    check(A, op=op, method=method)
    if op == "aat":
        check(A, op="aat_upper", method=method)


@pytest.fixture(scope="module")
def tier_matrix():
    return tier_matrix_rows()


@pytest.mark.parametrize("method", ["adaptive", "hash", "merge"])
def test_all_tiers(tier_matrix, method):
    C, st = check(tier_matrix, method=method)
    used = {k for k, v in st["tier_rows"].items() if v > 0}
    if method == "adaptive":
        assert {"rank2k", "hash64", "hash_block", "block_rank"} <= used, used
    if method == "hash":
        assert {"hash64", "hash_block", "window"} <= used, used
    if method == "merge":
        assert "merge" in used and "window" in used, used


@pytest.mark.parametrize("op", ["ab", "aat_upper"])
def test_block_rank_tier(op):
    A = hub_matrix()
    C, st = check(A, op=op)
    assert st["tier_rows"]["block_rank"] > 0, st["tier_rows"]


def test_handoff_arena_full_falls_back(monkeypatch):
    """Rows whose symbolic bitmap finds the handoff arena full rebuild it in the numeric phase;
    results are identical either way (and with no arena room at all)."""
    A = M.stencil27(g=24)
    monkeypatch.setenv("APPT_NO_SMALL_PATH", "1")
    C0 = ap.spgemm(A)
    for words in ("16384", "0"):
        monkeypatch.setenv("APPT_HANDOFF_WORDS", words)
        C1 = ap.spgemm(A)
        assert np.array_equal(C0.row_ptr, C1.row_ptr)
        assert np.array_equal(C0.col_idx, C1.col_idx)
        assert np.array_equal(C0.val, C1.val)
    R = oracle.spgemm(A)
    assert_same_structure(C0, R)
    assert np.array_equal(C0.val, R.val)


def test_host_results_views_and_pinned_reuse():
    """copy=False returns views of the library's pinned block; a released block is reused by
    the next host result without changing it."""
    A = M.stencil27(g=20)
    C = ap.spgemm(A, copy=False)
    R = oracle.spgemm(A)
    assert_same_structure(C, R)
    ci0 = C.col_idx.copy()
    del C
    for _ in range(3):
        C2 = ap.spgemm(A, copy=False)
        assert np.array_equal(C2.col_idx, ci0)
        del C2


def test_window_tier_dense_rows():
    """Rows of C with more than ~600 entries packed into at most 16384 columns take the dense
    window tier."""
    C, st = check(window_matrix())
    assert st["tier_rows"]["window"] > 0, st["tier_rows"]


def test_block_rank_multiwindow():
    """Rows of C spanning more than 2^20 columns are processed in several bitmap windows."""
    rng = np.random.default_rng(4)
    k, cols = 64, 1 << 22
    brows = [np.unique(rng.integers(0, cols, 3000)) for _ in range(k)]
    brp = np.zeros(k + 1, np.int64)
    brp[1:] = np.cumsum([len(r) for r in brows])
    bci = np.concatenate(brows).astype(np.int32)
    B = M.Csr(k, cols, brp.astype(np.int32), bci, rng.uniform(-1, 1, bci.size))
    A = M.random_csr(96, k, 0.25, 5)
    C, st = check(A, B)
    assert st["tier_rows"]["block_rank"] > 0, st["tier_rows"]


@pytest.mark.parametrize("op", ["ab", "ab_upper"])
def test_dense_b_rows_in_cta_symbolic_tier(op):
    """B rows with at least one entry per 32 columns are kept as bitmaps and ORed into the CTA
    symbolic tier's windows a word at a time. The rows of C span more than 2^20 columns (several
    windows, starts not aligned to 32), and A's rows mix dense and sparse B rows."""
    rng = np.random.default_rng(11)
    k, cols = 1024, (1 << 20) + 40000
    brows = [np.unique(rng.integers(0, cols, cols // 16 if r % 128 == 3 else 100))
             for r in range(k)]
    brp = np.zeros(k + 1, np.int64)
    brp[1:] = np.cumsum([len(r) for r in brows])
    bci = np.concatenate(brows).astype(np.int32)
    B = M.Csr(k, cols, brp.astype(np.int32), bci, rng.uniform(-1, 1, bci.size))
    m = 160
    arows = [np.unique(np.concatenate([rng.integers(0, k, 11), [128 * (r % 8) + 3]]))
             if r % 5 else np.unique(rng.integers(0, k, 12)) for r in range(m)]
    arp = np.zeros(m + 1, np.int64)
    arp[1:] = np.cumsum([len(r) for r in arows])
    aci = np.concatenate(arows).astype(np.int32)
    A = M.Csr(m, k, arp.astype(np.int32), aci, rng.uniform(-1, 1, aci.size))
    C, st = check(A, B, op=op)
    assert st["tier_rows"]["block_rank"] > 0, st["tier_rows"]


@pytest.mark.parametrize("cols", [1 << 22, 1 << 25])
@pytest.mark.parametrize("op", ["ab", "ab_upper"])
def test_cta_hash_tier_wide_spans(op, cols):
    """Rows of C with 513..2048 entries spread over millions of columns take the CTA hash tier
    (hash table sized from the exact nnz, compaction and an in-table sort)."""
    rng = np.random.default_rng(13)
    k = 64
    brows = [np.unique(rng.integers(0, cols, 100)) for _ in range(k)]
    brp = np.zeros(k + 1, np.int64)
    brp[1:] = np.cumsum([len(r) for r in brows])
    bci = np.concatenate(brows).astype(np.int32)
    B = M.Csr(k, cols, brp.astype(np.int32), bci, rng.uniform(-1, 1, bci.size))
    A = M.random_csr(200, k, 0.15, 6)
    C, st = check(A, B, op=op)
    assert st["tier_rows"]["hash_block"] > 0, st["tier_rows"]


@pytest.mark.parametrize("op", ["ab", "ab_upper"])
def test_dense_b_rows_in_window_tier(op):
    """Dense rows of C (window tier) built mostly from B rows kept as bitmaps: their products
    are added by per-warp column slices located through the bitmaps' popcount prefixes, the
    rest with shared atomics."""
    rng = np.random.default_rng(12)
    k, cols = 256, (1 << 17) + 5000
    brows = [np.unique(rng.integers(0, cols, cols // 7 if r % 32 == 5 else 200))
             for r in range(k)]
    brp = np.zeros(k + 1, np.int64)
    brp[1:] = np.cumsum([len(r) for r in brows])
    bci = np.concatenate(brows).astype(np.int32)
    B = M.Csr(k, cols, brp.astype(np.int32), bci, rng.uniform(-1, 1, bci.size))
    m = 100
    arows = [np.unique(np.concatenate([rng.integers(0, k, 5), 32 * rng.integers(0, 8, 3) + 5]))
             for _ in range(m)]
    arp = np.zeros(m + 1, np.int64)
    arp[1:] = np.cumsum([len(r) for r in arows])
    aci = np.concatenate(arows).astype(np.int32)
    A = M.Csr(m, k, arp.astype(np.int32), aci, rng.uniform(-1, 1, aci.size))
    C, st = check(A, B, op=op)
    assert st["tier_rows"]["window"] > 0, st["tier_rows"]


@pytest.mark.parametrize("method", ["adaptive", "hash", "esc"])
@pytest.mark.parametrize("name", ["uniform8", "stencil27", "banded", "random"])
def test_sequential_tiers_are_bit_exact(name, method):
    """The warp tiers (rank, warp hash) and ESC sum each column in the reference's k-then-j
    order with separate multiply and add roundings, so their values equal the oracle's bit for
    bit (the CTA tiers, used only for rows beyond 512 entries, accumulate with atomics)."""
    A = M.random_csr(2000, 2000, 0.005, 4) if name == "random" else M.make(name, small=True)
    C, st = ap.spgemm(A, method=method, return_stats=True)
    assert st["tier_rows"]["hash_block"] == 0 and st["tier_rows"]["window"] == 0
    assert st["tier_rows"]["block_rank"] == 0
    R = oracle.spgemm(A)
    assert_same_structure(C, R)
    assert np.array_equal(C.val, R.val)


def test_empty_and_degenerate():
    Z = M.Csr(0, 0, np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0))
    C = ap.spgemm(Z)
    assert C.rows == 0 and C.nnz == 0
    E = M.Csr(50, 50, np.zeros(51, np.int32), np.zeros(0, np.int32), np.zeros(0))
    for method in METHODS:
        C = ap.spgemm(E, method=method)
        assert C.nnz == 0 and C.rows == 50
    one = M.Csr(1, 1, np.array([0, 1], np.int32), np.array([0], np.int32), np.array([3.0]))
    C = ap.spgemm(one)
    assert C.nnz == 1 and C.val[0] == 9.0
    # a single dense row hitting every column, plus an identity
    n = 3000
    rp = np.concatenate([[0, n], n + np.arange(1, n)]).astype(np.int32)
    ci = np.concatenate([np.arange(n), np.arange(1, n)]).astype(np.int32)
    D = M.Csr(n, n, rp, ci, np.random.default_rng(0).uniform(-1, 1, ci.size))
    for method in METHODS:
        check(D, method=method)


def test_cancellation_keeps_structural_zeros():
    # row 0 of A = e0 - e1 and rows 0, 1 of B are equal -> row 0 of C sums to exact zeros,
    # which stay stored; row 1 of A = e0 + e2 reaches columns {1, 2} u {0}.
    A = M.Csr(3, 3, np.array([0, 2, 4, 5], np.int32), np.array([0, 1, 0, 2, 2], np.int32),
              np.array([1.0, -1.0, 1.0, 1.0, 1.0]))
    B = M.Csr(3, 3, np.array([0, 2, 4, 5], np.int32), np.array([1, 2, 1, 2, 0], np.int32),
              np.array([2.0, 3.0, 2.0, 3.0, 1.0]))
    for method in METHODS:
        C = ap.spgemm(A, B, method=method)
        R = oracle.spgemm(A, B)
        assert_same_structure(C, R)
        assert C.nnz == R.nnz == 6
        assert np.array_equal(C.row_ptr, [0, 2, 5, 6])
        assert np.array_equal(C.val[:2], [0.0, 0.0])
        assert np.array_equal(C.val[2:], [1.0, 2.0, 3.0, 1.0])


def test_invalid_column_is_an_error_not_a_fault():
    A = M.Csr(4, 4, np.array([0, 1, 2, 3, 4], np.int32), np.array([0, 9, 2, 3], np.int32),
              np.ones(4))
    with pytest.raises(ap.ApptError):
        ap.spgemm(A)
    # the context is still usable afterwards
    check(M.random_csr(64, 64, 0.1, 3))


def test_host_row_block_operand():
    """A host row block (row_ptr not starting at 0, global col_idx/val) multiplies like the
    corresponding rows of the full product."""
    A = M.random_csr(500, 500, 0.03, 17, empty_rows=0.1)
    r0, r1 = 137, 401
    blk = M.Csr(r1 - r0, A.cols, A.row_ptr[r0:r1 + 1], A.col_idx, A.val)
    C = ap.spgemm(blk, A)
    R = oracle.spgemm(A)
    lo, hi = int(R.row_ptr[r0]), int(R.row_ptr[r1])
    assert np.array_equal(C.row_ptr, R.row_ptr[r0:r1 + 1] - lo)
    assert np.array_equal(C.col_idx, R.col_idx[lo:hi])
    assert np.array_equal(C.val, R.val[lo:hi])


def test_uniform8_full():
    check(M.uniform8())


def test_stencil27_full():
    check(M.stencil27())


def test_banded_quarter_full():
    check(M.banded(n=1 << 20))


def test_transpose_matches_oracle():
    A = M.zipf_att(rows=1 << 14, cols=1 << 12)
    T = ap.transpose(A)
    R = oracle.transpose(A)
    assert np.array_equal(T.row_ptr, R.row_ptr.astype(np.int64))
    assert np.array_equal(T.col_idx, R.col_idx)
    assert np.array_equal(T.val, R.val)


def test_row_products_match_oracle():
    A = M.rmat(scale=14)
    assert np.array_equal(ap.row_products(A), oracle.row_products(A))


@pytest.mark.parametrize("estimator", ["minhash", "hll"])
@pytest.mark.parametrize("att", [False, True])
def test_estimator_matches_reference_restatement(att, estimator):
    small = M.random_csr(500, 500, 0.02, 9)                   # nnz < 100000: products count
    big = M.stencil27(g=24)                                   # nnz >= 100000: the sketches
    for A in (small, big):
        e = ap.estimate_row_nnz(A, att=att, estimator=estimator)
        r = oracle.estimate_row_nnz(A, att=att, estimator=estimator)
        assert e.shape == r.shape
        # the only floating-point steps that can differ between the device and the host are
        # the final log/division, so at most isolated rows may snap differently
        assert (e != r).sum() <= max(1, A.rows // 10000), int((e != r).sum())


def test_estimator_env_selection(monkeypatch):
    """EST_METHOD=hll selects HyperLogLog for the default estimator, as in the reference."""
    A = M.stencil27(g=24)
    monkeypatch.setenv("EST_METHOD", "hll")
    e = ap.estimate_row_nnz(A)
    assert np.array_equal(e, ap.estimate_row_nnz(A, estimator="hll"))


def test_reference_score_matches_restatement():
    for name in M.WORKLOADS:
        A = M.make(name, small=True)
        assert abs(ap.reference_score(A) - oracle.reference_score(A)) < 1e-12
