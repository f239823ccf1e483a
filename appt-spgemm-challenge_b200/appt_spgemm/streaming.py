"""Row-block streaming for products whose C does not fit in device memory.

C = A*A^T of the 2^18 x 2^16 Zipf workload is ~99% dense: about 6.8e10 entries, ~817 GB, more
than one GPU (or four) holds. Rows of C are independent, so the product is computed as a
sequence of row blocks against a device-resident B (= A^T, built once on the device), each block
handed to a consumer and released before the next one. Blocks are cut so that their
intermediate products (an upper bound of their nnz) stay under a budget.

The per-block work is the engine's device-operand call (appt_spgemm with APPT_MEM_DEVICE
operands, APPT_OP_AB or APPT_OP_AB_UPPER with row_base); nothing here computes on the CPU.
"""
from __future__ import annotations

from typing import Callable

import numpy as np

from . import DeviceResult, spgemm_device


def row_products_aat(A) -> np.ndarray:
    """Intermediate products per row of A*A^T: sum over the row's columns k of count(k)."""
    counts = np.bincount(np.asarray(A.col_idx, np.int64), minlength=A.cols)
    per_entry = counts[np.asarray(A.col_idx, np.int64)]
    rp = np.asarray(A.row_ptr, np.int64)
    out = np.zeros(A.rows, np.int64)
    nz = rp[1:] > rp[:-1]
    if per_entry.size:
        sums = np.add.reduceat(per_entry, rp[:-1][nz])
        out[nz] = sums
    return out


def cut_blocks(row_products: np.ndarray, max_products: int, max_rows: int | None = None):
    """Contiguous row blocks whose products sum stays <= max_products (a row larger than the
    budget forms a block of its own)."""
    bounds = [0]
    acc = 0
    start = 0
    for i, p in enumerate(np.asarray(row_products, np.int64).tolist()):
        if i > start and (acc + p > max_products or (max_rows and i - start >= max_rows)):
            bounds.append(i)
            start = i
            acc = 0
        acc += p
    bounds.append(len(row_products))
    if bounds[-2] == bounds[-1]:
        bounds.pop()
    return bounds


def stream_row_blocks(A, a_dev: tuple, b_dev: tuple, bounds, consume: Callable[[int, int,
                      DeviceResult], None], upper: bool = False, stream: int | None = None,
                      device: int = 0, method: str = "adaptive") -> dict:
    """Compute C = A*B block by block. a_dev = (row_ptr, col_idx, val) device pointers of A
    (int32/int32/fp64), b_dev = (rows, cols, nnz, row_ptr, col_idx, val) of B on the device.
    consume(r0, r1, result) sees each block's device C before it is freed. Returns totals."""
    rp_host = np.asarray(A.row_ptr, np.int64)
    total_nnz = 0
    total_products = 0
    for r0, r1 in zip(bounds[:-1], bounds[1:]):
        blk_nnz = int(rp_host[r1] - rp_host[r0])
        res = spgemm_device(r1 - r0, A.cols, blk_nnz, a_dev[0] + 4 * r0, a_dev[1], a_dev[2],
                            B=b_dev, op="ab_upper" if upper else "ab", row_base=r0,
                            stream=stream, device=device, method=method)
        try:
            total_nnz += res.nnz
            total_products += res.stats["products"]
            consume(r0, r1, res)
        finally:
            res.free()
    return {"nnz": total_nnz, "products": total_products, "blocks": len(bounds) - 1}
