"""Seeded synthetic CSR inputs (numpy PCG64) for the five benchmark workloads.

The reference measures on SuiteSparse matrices that are not available offline; these
generators stand in for them with the shapes, sizes and value distributions of the
benchmark workloads:

  uniform8   n=4096, exactly 8 distinct uniform columns per row, vals U(-1,1), seed 0, C=A*A
  stencil27  27-point stencil on a g^3 grid (g=64), boundary rows truncated, vals U(0.5,1.5),
             seed 1, C=A*A
  rmat       R-MAT n=2^scale (scale 20), 16*n edges, (a,b,c,d)=(.57,.19,.19,.05), duplicates
             merged, self-loops kept, vals U(0,1), seed 2, C=A*A
  zipf_att   2^18 x 2^16, 32 distinct columns per row drawn Zipf(s=1.1) over a seeded
             permutation of column ids, vals U(-1,1), seed 3, C=A*A^T
  banded     n=2^22, 16 distinct columns per row uniform within +-256 of the diagonal,
             vals U(-1,1), seed 4, C=A*A

Every generator takes size parameters so tests can build small instances of the same family.
Columns are sorted inside every row; row_ptr/col_idx are int32 and values fp64.
"""
from __future__ import annotations

import dataclasses
import struct
from pathlib import Path

import numpy as np


@dataclasses.dataclass
class Csr:
    rows: int
    cols: int
    row_ptr: np.ndarray   # int32 (inputs) or int64 (results), rows + 1
    col_idx: np.ndarray   # int32
    val: np.ndarray       # float64

    @property
    def nnz(self) -> int:
        return int(self.row_ptr[-1] - self.row_ptr[0])

    def row_lengths(self) -> np.ndarray:
        return np.diff(self.row_ptr.astype(np.int64))

    def to_scipy(self):
        import scipy.sparse as sp
        return sp.csr_matrix((self.val, self.col_idx, self.row_ptr.astype(np.int64)),
                             shape=(self.rows, self.cols))

    @staticmethod
    def from_scipy(m) -> "Csr":
        m = m.tocsr()
        m.sort_indices()
        return Csr(m.shape[0], m.shape[1], m.indptr.astype(np.int32), m.indices.astype(np.int32),
                   m.data.astype(np.float64))


def _distinct_sorted_rows(rng, rows: int, per_row: int, draw) -> np.ndarray:
    """Draw `per_row` distinct values per row via `draw(rng, n_rows, k)`; redraw rows with
    duplicates until none remain. Returns a sorted (rows, per_row) int64 array."""
    out = np.sort(draw(rng, np.arange(rows), per_row), axis=1)
    bad = np.nonzero((np.diff(out, axis=1) == 0).any(axis=1))[0]
    while bad.size:
        redo = np.sort(draw(rng, bad, per_row), axis=1)
        out[bad] = redo
        bad = bad[(np.diff(redo, axis=1) == 0).any(axis=1)]
    return out


def _from_dense_rows(rows: int, cols: int, colmat: np.ndarray, vals: np.ndarray) -> Csr:
    per = colmat.shape[1]
    rp = (np.arange(rows + 1, dtype=np.int64) * per).astype(np.int32)
    return Csr(rows, cols, rp, colmat.reshape(-1).astype(np.int32), vals.astype(np.float64))


def uniform8(n: int = 4096, per_row: int = 8, seed: int = 0) -> Csr:
    rng = np.random.default_rng(seed)
    cols = _distinct_sorted_rows(rng, n, per_row,
                                 lambda r, idx, k: r.integers(0, n, size=(len(idx), k)))
    vals = rng.uniform(-1.0, 1.0, size=n * per_row)
    return _from_dense_rows(n, n, cols, vals)


def stencil27(g: int = 64, seed: int = 1, gz: int | None = None) -> Csr:
    """27-point stencil on a g x g x gz grid (gz defaults to g); row i = (z*g + y)*g + x;
    neighbours outside the grid are dropped (boundary truncation)."""
    rng = np.random.default_rng(seed)
    gz = g if gz is None else gz
    n = g * g * gz
    idx = np.arange(n, dtype=np.int64)
    x, y, z = idx % g, (idx // g) % g, idx // (g * g)
    cols = []
    masks = []
    for dz in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dx in (-1, 0, 1):
                ok = ((x + dx >= 0) & (x + dx < g) & (y + dy >= 0) & (y + dy < g) &
                      (z + dz >= 0) & (z + dz < gz))
                cols.append(idx + dx + g * dy + g * g * dz)
                masks.append(ok)
    C = np.stack(cols, axis=1)          # offsets in increasing order -> sorted columns
    M = np.stack(masks, axis=1)
    counts = M.sum(axis=1)
    rp = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts, out=rp[1:])
    ci = C[M]
    vals = rng.uniform(0.5, 1.5, size=ci.size)
    return Csr(n, n, rp.astype(np.int32), ci.astype(np.int32), vals)


def rmat(scale: int = 20, edge_factor: int = 16, a: float = 0.57, b: float = 0.19,
         c: float = 0.19, seed: int = 2) -> Csr:
    rng = np.random.default_rng(seed)
    n = 1 << scale
    E = edge_factor * n
    r = np.zeros(E, dtype=np.int64)
    cc = np.zeros(E, dtype=np.int64)
    ab, abc = a + b, a + b + c
    for lvl in range(scale):
        u = rng.random(E)
        rowbit = u >= ab
        colbit = ((u >= a) & (u < ab)) | (u >= abc)
        r |= rowbit.astype(np.int64) << lvl
        cc |= colbit.astype(np.int64) << lvl
    key = np.unique(r * n + cc)          # merge duplicates; self-loops kept
    rows = key // n
    cols = key % n
    counts = np.bincount(rows, minlength=n)
    rp = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts, out=rp[1:])
    vals = rng.random(key.size)
    return Csr(n, n, rp.astype(np.int32), cols.astype(np.int32), vals)


def zipf_att(rows: int = 1 << 18, cols: int = 1 << 16, per_row: int = 32, s: float = 1.1,
             seed: int = 3) -> Csr:
    """Rows of `per_row` distinct columns drawn from Zipf(s) over ranks 1..cols, mapped through
    a seeded permutation of column ids."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(cols)
    w = 1.0 / np.power(np.arange(1, cols + 1, dtype=np.float64), s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]

    def draw_distinct(idx_rows: np.ndarray) -> np.ndarray:
        out = np.empty((len(idx_rows), per_row), dtype=np.int64)
        pending = np.arange(len(idx_rows))
        extra = 4 * per_row
        while pending.size:
            d = np.searchsorted(cdf, rng.random((pending.size, extra)), side="right")
            d = np.minimum(d, cols - 1)
            # first per_row distinct ranks of each row, in draw order
            order = np.argsort(d, axis=1, kind="stable")
            ds = np.take_along_axis(d, order, axis=1)
            first = np.ones_like(ds, dtype=bool)
            first[:, 1:] = ds[:, 1:] != ds[:, :-1]
            keep_pos = np.where(first, order, extra)        # position of first occurrences
            keep_pos.sort(axis=1)
            ok = keep_pos[:, per_row - 1] < extra
            got = np.take_along_axis(d, np.minimum(keep_pos[:, :per_row], extra - 1), axis=1)
            out[pending[ok]] = got[ok]
            pending = pending[~ok]
        return out

    ranks = np.concatenate([draw_distinct(np.arange(lo, min(lo + 65536, rows)))
                            for lo in range(0, rows, 65536)])
    colmat = np.sort(perm[ranks], axis=1)
    vals = rng.uniform(-1.0, 1.0, size=rows * per_row)
    return _from_dense_rows(rows, cols, colmat, vals)


def banded(n: int = 1 << 22, per_row: int = 16, half_width: int = 256, seed: int = 4) -> Csr:
    rng = np.random.default_rng(seed)

    def draw(r, idx, k):
        lo = np.maximum(idx - half_width, 0)
        hi = np.minimum(idx + half_width, n - 1)
        span = (hi - lo + 1)[:, None]
        return lo[:, None] + (r.random((len(idx), k)) * span).astype(np.int64)

    out = np.empty((n, per_row), dtype=np.int64)
    step = 1 << 20
    for s0 in range(0, n, step):
        idx = np.arange(s0, min(s0 + step, n))
        cols = np.sort(draw(rng, idx, per_row), axis=1)
        bad = np.nonzero((np.diff(cols, axis=1) == 0).any(axis=1))[0]
        while bad.size:
            redo = np.sort(draw(rng, idx[bad], per_row), axis=1)
            cols[bad] = redo
            bad = bad[(np.diff(redo, axis=1) == 0).any(axis=1)]
        out[s0:s0 + len(idx)] = cols
    vals = rng.uniform(-1.0, 1.0, size=n * per_row)
    return _from_dense_rows(n, n, out, vals)


def random_csr(rows: int, cols: int, density: float, seed: int, empty_rows: float = 0.0,
               value_range=(-1.0, 1.0)) -> Csr:
    """Small random CSR for tests (Bernoulli pattern, optional forced empty rows)."""
    rng = np.random.default_rng(seed)
    mask = rng.random((rows, cols)) < density
    if empty_rows > 0:
        mask[rng.random(rows) < empty_rows] = False
    r, c = np.nonzero(mask)
    counts = np.bincount(r, minlength=rows)
    rp = np.zeros(rows + 1, dtype=np.int64)
    np.cumsum(counts, out=rp[1:])
    vals = rng.uniform(value_range[0], value_range[1], size=r.size)
    return Csr(rows, cols, rp.astype(np.int32), c.astype(np.int32), vals)


# Workload table: name -> (generator, op, full-size kwargs, small-size kwargs)
WORKLOADS = {
    "uniform8": (uniform8, "ab", {}, {"n": 512}),
    "stencil27": (stencil27, "ab", {}, {"g": 12}),
    "rmat": (rmat, "ab", {}, {"scale": 10}),
    "zipf_att": (zipf_att, "aat", {}, {"rows": 2048, "cols": 512}),
    "banded": (banded, "ab", {}, {"n": 1 << 12}),
}


def make(name: str, small: bool = False, **overrides) -> Csr:
    gen, _op, full, smallkw = WORKLOADS[name]
    kw = dict(smallkw if small else full)
    kw.update(overrides)
    return gen(**kw)


# ----------------------------------------------------------------------------- binary CSR files
_MAGIC = b"APPTCSR1"


def save_bin(path, A: Csr) -> None:
    """Binary CSR: magic, int64 rows/cols/nnz, int32 row_ptr, int32 col_idx, f64 val."""
    with open(path, "wb") as f:
        f.write(_MAGIC)
        f.write(struct.pack("<qqq", A.rows, A.cols, A.nnz))
        f.write(np.ascontiguousarray(A.row_ptr, dtype=np.int32).tobytes())
        f.write(np.ascontiguousarray(A.col_idx, dtype=np.int32).tobytes())
        f.write(np.ascontiguousarray(A.val, dtype=np.float64).tobytes())


def load_bin(path) -> Csr:
    data = Path(path).read_bytes()
    if data[:8] != _MAGIC:
        raise ValueError(f"{path}: not an APPTCSR1 file")
    rows, cols, nnz = struct.unpack_from("<qqq", data, 8)
    off = 32
    rp = np.frombuffer(data, dtype=np.int32, count=rows + 1, offset=off)
    off += 4 * (rows + 1)
    ci = np.frombuffer(data, dtype=np.int32, count=nnz, offset=off)
    off += 4 * nnz
    val = np.frombuffer(data, dtype=np.float64, count=nnz, offset=off)
    return Csr(rows, cols, rp.copy(), ci.copy(), val.copy())
