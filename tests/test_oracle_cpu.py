"""The CPU oracle against independent implementations (pure Python, scipy) and known answers."""
import numpy as np
import pytest
import scipy.sparse as sp

import oracle
from appt_spgemm import matrices as M


def murmur3_32(data: bytes, seed: int) -> int:
    """Generic MurmurHash3_x86_32 (Austin Appleby's published algorithm), independent of
    oracle.c's 4-byte specialisation."""
    c1, c2 = 0xCC9E2D51, 0x1B873593
    h = seed & 0xFFFFFFFF
    n = len(data)
    rotl = lambda x, r: ((x << r) | (x >> (32 - r))) & 0xFFFFFFFF  # noqa: E731
    for i in range(0, n - n % 4, 4):
        k = int.from_bytes(data[i:i + 4], "little")
        k = (k * c1) & 0xFFFFFFFF
        k = rotl(k, 15)
        k = (k * c2) & 0xFFFFFFFF
        h ^= k
        h = rotl(h, 13)
        h = (h * 5 + 0xE6546B64) & 0xFFFFFFFF
    tail = data[n - n % 4:]
    k = 0
    if len(tail) >= 3:
        k ^= tail[2] << 16
    if len(tail) >= 2:
        k ^= tail[1] << 8
    if len(tail) >= 1:
        k ^= tail[0]
        k = (k * c1) & 0xFFFFFFFF
        k = rotl(k, 15)
        k = (k * c2) & 0xFFFFFFFF
        h ^= k
    h ^= n
    h ^= h >> 16
    h = (h * 0x85EBCA6B) & 0xFFFFFFFF
    h ^= h >> 13
    h = (h * 0xC2B2AE35) & 0xFFFFFFFF
    h ^= h >> 16
    return h


@pytest.mark.parametrize("data,seed,want", [
    (b"", 0, 0x00000000),
    (b"", 1, 0x514E28B7),
    (b"", 0xFFFFFFFF, 0x81F16F39),
    (b"\x00\x00\x00\x00", 0, 0x2362F9DE),
    (b"aaaa", 0x9747B28C, 0x5A97808A),
    (b"Hello, world!", 0x9747B28C, 0x24884CBA),
])
def test_murmur3_published_vectors(data, seed, want):
    assert murmur3_32(data, seed) == want


def test_oracle_murmur3_matches_generic_with_reference_seed():
    rng = np.random.default_rng(0)
    for key in [0, 1, 2, 0x7FFFFFFF, 0xFFFFFFFF] + rng.integers(0, 2**31, 200).tolist():
        assert oracle.murmur3(int(key)) == murmur3_32(int(key).to_bytes(4, "little"), 1234)


@pytest.mark.parametrize("seed", range(4))
def test_oracle_matches_pure_python(seed):
    A = M.random_csr(60, 60, 0.08, seed, empty_rows=0.1)
    C = oracle.spgemm(A)
    rp, cols, vals = oracle.spgemm_py(A)
    assert np.array_equal(C.row_ptr, rp)
    assert np.array_equal(C.col_idx, cols)
    assert np.array_equal(C.val, vals)          # same summation order: bit-exact
    Cu = oracle.spgemm(A, op="aat_upper")
    T = oracle.transpose(A)
    rp, cols, vals = oracle.spgemm_py(A, T, upper=True)
    assert np.array_equal(Cu.row_ptr, rp) and np.array_equal(Cu.col_idx, cols)
    assert np.array_equal(Cu.val, vals)


@pytest.mark.parametrize("name", list(M.WORKLOADS))
def test_oracle_matches_scipy(name):
    A = M.make(name, small=True)
    op = M.WORKLOADS[name][1]
    S = A.to_scipy()
    R = (S @ S.T) if op == "aat" else (S @ S)
    P = (abs(S) @ abs(S).T) if op == "aat" else (abs(S) @ abs(S))   # no cancellation: pattern
    C = oracle.spgemm(A, op=op)
    P.sort_indices()
    assert np.array_equal(C.row_ptr, P.indptr) and np.array_equal(C.col_idx, P.indices)
    D = sp.csr_matrix((C.val, C.col_idx, C.row_ptr), shape=R.shape)
    diff = abs(D - R).max() if R.nnz else 0.0
    assert diff <= 1e-12 * max(1.0, abs(P).max())


def test_oracle_transpose_matches_scipy():
    A = M.zipf_att(rows=4096, cols=1024)
    T = oracle.transpose(A)
    S = A.to_scipy().T.tocsr()
    S.sort_indices()
    assert np.array_equal(T.row_ptr, S.indptr) and np.array_equal(T.col_idx, S.indices)
    assert np.array_equal(T.val, S.data)


def test_upper_triangle_identity_on_symmetric_input():
    """For symmetric A with a full diagonal, nnz(upper(A*A^T)) = (nnz(A*A) + n) / 2 -- the
    reference's algebraic cross-check for the att paths."""
    A = M.stencil27(g=10)
    full = oracle.spgemm(A)
    up = oracle.spgemm(A, op="aat_upper")
    diag = sum(1 for i in range(A.rows)
               if i in set(full.col_idx[full.row_ptr[i]:full.row_ptr[i + 1]].tolist()))
    assert up.nnz == (full.nnz + diag) // 2


def test_row_products_and_estimate_small_path():
    A = M.random_csr(200, 200, 0.05, 3)
    f = oracle.row_products(A)
    S = A.to_scipy()
    lens = np.diff(S.indptr)
    assert np.array_equal(f, np.array([lens[S.indices[S.indptr[i]:S.indptr[i + 1]]].sum()
                                       for i in range(A.rows)]))
    assert np.array_equal(oracle.estimate_row_nnz(A), f.astype(np.int32))


def test_minhash_estimate_properties():
    A = M.stencil27(g=24)           # nnz >= 100000: the MinHash path
    est = oracle.estimate_row_nnz(A)
    exact = oracle.symbolic_counts(A)
    snapped = (est <= 16) | ((est & (est - 1)) == 0)
    assert snapped.all()
    assert est.min() >= 1 and est.max() <= 16384
    # x1.5 expansion keeps the estimate at or above the exact count for most rows
    assert np.mean(est >= exact) > 0.95


def _hll_estimate_py(A, B):
    """Pure-Python HyperLogLog estimate (the algorithm of the reference's hll_construct_kernel
    / hll_merge_kernel): independent of oracle.c."""
    import math
    brp, bci = np.asarray(B.row_ptr, np.int64), np.asarray(B.col_idx)
    regs = np.zeros((B.rows, 128), np.uint8)
    for r in range(B.rows):
        for c in bci[brp[r]:brp[r + 1]]:
            h = murmur3_32(int(c).to_bytes(4, "little"), 1234)
            rho = min(33 - h.bit_length(), 26) if h else 26
            regs[r, h & 127] = max(regs[r, h & 127], rho)
    arp, aci = np.asarray(A.row_ptr, np.int64), np.asarray(A.col_idx)
    out = np.zeros(A.rows, np.int32)
    for i in range(A.rows):
        mx = regs[aci[arp[i]:arp[i + 1]]].max(axis=0) if arp[i + 1] > arp[i] else regs[0] * 0
        z = sum(1.0 / float(1 << int(v)) for v in mx)
        empty = int((mx == 0).sum())
        E = 0.715 * 128.0 * 128.0 / z
        if empty and E <= 2.5 * 128:
            E = 128.0 * math.log(128.0 / empty)
        t = max(int(E * 1.5), 1)
        if t > 16:
            ht = 32
            while ht < t and ht < 16384:
                ht <<= 1
            t = ht
        out[i] = t
    return out


def test_hll_estimate_matches_python_restatement():
    A = M.stencil27(g=24)           # nnz >= 100000: the sketch path
    est = oracle.estimate_row_nnz(A, estimator="hll")
    rows = np.arange(0, A.rows, 97)
    sub = M.Csr(len(rows), A.cols, np.concatenate([[0], np.cumsum(np.diff(A.row_ptr)[rows])]).astype(np.int32),
                np.concatenate([A.col_idx[A.row_ptr[r]:A.row_ptr[r + 1]] for r in rows]),
                np.concatenate([A.val[A.row_ptr[r]:A.row_ptr[r + 1]] for r in rows]))
    assert np.array_equal(est[rows], _hll_estimate_py(sub, A))
    exact = oracle.symbolic_counts(A)
    assert np.mean(est >= exact) > 0.9


def test_reference_score_known_choices():
    """The reference dispatcher sends the small uniform workload to merge3 and the stencil to
    hash (score sign)."""
    assert oracle.reference_score(M.uniform8()) > 0
    assert oracle.reference_score(M.stencil27(g=32)) < 0
