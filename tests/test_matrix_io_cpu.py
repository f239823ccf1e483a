"""Matrix files for the reference's driver (the library's read_matrix_market / write_matrix_market,
include/spgemm.h:44-52 of the reference), on the CPU: MatrixMarket text in its banner variants
and the binary CSR form read into the reference's single-buffer layout, against independent
parses; and the reference's src/main.cu linked against the library (built by build() when the
reference sources are present).
"""
import ctypes as ct
import subprocess

import numpy as np
import pytest

import appt_spgemm as ap
from appt_spgemm import matrices as M


def _read(path):
    lib = ap.load()
    fn = lib.appt_read_matrix_file
    fn.argtypes = [ct.c_char_p, ct.POINTER(ct.c_void_p), ct.POINTER(ct.c_void_p),
                   ct.POINTER(ct.c_void_p), ct.POINTER(ct.c_void_p), ct.POINTER(ct.c_int),
                   ct.POINTER(ct.c_int), ct.POINTER(ct.c_int)]
    fn.restype = ct.c_bool
    buf, rp, ci, va = ct.c_void_p(), ct.c_void_p(), ct.c_void_p(), ct.c_void_p()
    r, c, n = ct.c_int(), ct.c_int(), ct.c_int()
    ok = fn(str(path).encode(), ct.byref(buf), ct.byref(rp), ct.byref(ci), ct.byref(va),
            ct.byref(r), ct.byref(c), ct.byref(n))
    if not ok:
        return None
    rows, nnz = r.value, n.value
    # the reference's layout: row_ptr | col_idx | pad to 8 | val, one block
    assert ci.value == buf.value + 4 * (rows + 1)
    assert va.value == buf.value + ((4 * (rows + 1) + 4 * nnz + 7) & ~7)
    A = M.Csr(rows, c.value,
              np.ctypeslib.as_array(ct.cast(rp, ct.POINTER(ct.c_int32)), (rows + 1,)).copy(),
              np.ctypeslib.as_array(ct.cast(ci, ct.POINTER(ct.c_int32)), (max(nnz, 1),))[:nnz].copy(),
              np.ctypeslib.as_array(ct.cast(va, ct.POINTER(ct.c_double)), (max(nnz, 1),))[:nnz].copy())
    lib.host_free.argtypes = [ct.c_void_p]
    lib.host_free(buf)
    return A


def _write(path, A):
    lib = ap.load()
    fn = lib.appt_write_matrix_file
    fn.argtypes = [ct.c_char_p, ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int,
                   ct.c_int]
    fn.restype = ct.c_bool
    rp = np.ascontiguousarray(A.row_ptr, np.int32)
    ci = np.ascontiguousarray(A.col_idx, np.int32)
    va = np.ascontiguousarray(A.val, np.float64)
    assert fn(str(path).encode(), rp.ctypes.data, ci.ctypes.data, va.ctypes.data, A.rows, A.cols,
              A.nnz)


def _same(A, B):
    assert (A.rows, A.cols, A.nnz) == (B.rows, B.cols, B.nnz)
    assert np.array_equal(np.asarray(A.row_ptr, np.int64), np.asarray(B.row_ptr, np.int64))
    assert np.array_equal(A.col_idx, B.col_idx)
    assert np.array_equal(A.val, B.val)


def _expected(rows, cols, entries):
    """CSR of (r, c, v) triples (0-based), rows sorted by (column, value)."""
    per = [[] for _ in range(rows)]
    for r, c, v in entries:
        per[r].append((c, v))
    rp, ci, va = [0], [], []
    for row in per:
        for c, v in sorted(row):
            ci.append(c)
            va.append(v)
        rp.append(len(ci))
    return M.Csr(rows, cols, np.array(rp, np.int32), np.array(ci, np.int32),
                 np.array(va, np.float64))


@pytest.mark.parametrize("kind", ["general", "symmetric", "pattern", "complex"])
def test_matrix_market_text(tmp_path, kind):
    rng = np.random.default_rng(3)
    rows, cols = (40, 40) if kind == "symmetric" else (37, 53)
    cells = set()
    while len(cells) < 200:
        r, c = int(rng.integers(rows)), int(rng.integers(cols))
        if kind == "symmetric" and c > r:
            r, c = c, r
        cells.add((r, c))
    cells = list(cells)
    rng.shuffle(cells)   # entries in no particular order, as files often are
    vals = rng.uniform(-10, 10, len(cells)).round(6)
    lines = [f"%%MatrixMarket matrix coordinate "
             f"{'pattern' if kind == 'pattern' else 'complex' if kind == 'complex' else 'real'} "
             f"{'symmetric' if kind == 'symmetric' else 'general'}", "% a comment",
             f"{rows} {cols} {len(cells)}"]
    entries = []
    for (r, c), v in zip(cells, vals.tolist()):
        if kind == "pattern":
            lines.append(f"{r + 1} {c + 1}")
            v = 1.0
        elif kind == "complex":
            lines.append(f"{r + 1} {c + 1} {v!r} 0.5")
        else:
            lines.append(f"{r + 1}\t{c + 1}  {'+' if v > 0 else ''}{v!r}")
        entries.append((r, c, float(v)))
        if kind == "symmetric" and r != c:
            entries.append((c, r, float(v)))
    p = tmp_path / "a.mtx"
    p.write_text("\n".join(lines) + "\n")
    _same(_read(p), _expected(rows, cols, entries))


def test_binary_round_trip_and_writer(tmp_path):
    A = M.random_csr(500, 300, 0.02, 9, empty_rows=0.1)
    p = tmp_path / "a.bin"
    M.save_bin(p, A)
    _same(_read(p), A)
    q = tmp_path / "b.bin"
    _write(q, A)                       # the writer's binary form reads back exactly
    _same(_read(q), A)
    t = tmp_path / "c.mtx"
    _write(t, A)                       # the reference's text form: %g values
    B = _read(t)
    assert np.array_equal(B.col_idx, A.col_idx)
    assert np.allclose(B.val, A.val, rtol=1e-5, atol=0)


def test_unreadable_inputs_fail_cleanly(tmp_path):
    assert _read(tmp_path / "missing.mtx") is None
    bad = tmp_path / "bad.mtx"
    bad.write_text("%%MatrixMarket matrix coordinate real general\n3 3 2\n1 1 1.0\n9 9 2.0\n")
    assert _read(bad) is None


def test_reference_driver_links_against_the_library():
    """build() links the reference's src/main.cu against libappt_spgemm.so (no reference kernel
    objects, no src/matrix_utils.cu). Skipped when the reference sources were not present at
    build time."""
    drv = ap.PKG_DIR / "_build" / "spgemm_test"
    if not drv.exists():
        pytest.skip("reference driver not built (reference sources absent)")
    out = subprocess.run(["ldd", str(drv)], capture_output=True, text=True).stdout
    assert "libappt_spgemm.so" in out and "not found" not in out
    syms = subprocess.run(["nm", "-D", "--undefined-only", "-C", str(drv)], capture_output=True,
                          text=True).stdout
    for name in ("spgemm_self_product_adaptive", "read_matrix_market", "pinned_free"):
        assert name in syms, name
