"""Row-sharded multi-GPU SpGEMM: Python side of the library's multi-GPU C ABI (appt_comm_*).

The reference is single-GPU (src/main.cu:44 selects device 0). Here rows of A are independent
units: one process per GPU computes a contiguous block of rows of C, the blocks balanced by
intermediate-product count; B (or A^T) is replicated to every GPU once with NCCL broadcasts, and
each product does one all-gather of the ranks' nnz(C block), from which every rank derives the
global offset of its block. C stays sharded. All of that runs inside libappt_spgemm.so (C++ over
NCCL, loaded at run time); this module only marshals arguments. Exchanging the 128-byte
communicator id between processes is the caller's business (any host channel).

Host-only helpers (split_rows, block_offsets, assemble_blocks) need no GPU.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from . import (B_DEVICE, CsrIn, CsrOut, DeviceResult, MEM_DEVICE, MEM_HOST, Stats, _check,
               _options, _take_host_out, _view_host_out, load)
from .matrices import Csr

ID_BYTES = 128


def split_rows(row_products, parts: int) -> list[int]:
    """Contiguous row bounds [0 = b_0, b_1, ..., b_parts = rows] that split the per-row
    intermediate products as evenly as contiguous blocks allow (appt_split_rows)."""
    p = np.ascontiguousarray(row_products, dtype=np.int64)
    out = np.zeros(int(parts) + 1, dtype=np.int64)
    _check(load().appt_split_rows(p.ctypes.data if p.size else None, p.size, int(parts),
                                  out.ctypes.data), "appt_split_rows")
    return [int(x) for x in out]


partition_rows = split_rows


def block_offsets(nnz_per_rank) -> np.ndarray:
    """Exclusive prefix of the ranks' nnz(C block): the global offset of each block's first
    entry (int64), plus the total as the last element."""
    v = np.asarray(nnz_per_rank, dtype=np.int64)
    out = np.zeros(v.size + 1, dtype=np.int64)
    np.cumsum(v, out=out[1:])
    return out


def global_row_ptr(local_row_ptr: np.ndarray, offset: int) -> np.ndarray:
    """Row pointers of a block shifted to global entry positions."""
    return np.asarray(local_row_ptr, dtype=np.int64) + int(offset)


def assemble_blocks(bounds, cols: int, blocks, offsets) -> Csr:
    """The whole C from the ranks' host blocks (each a Csr whose row_ptr starts at 0), in rank
    order, placed at `offsets` (block_offsets of the ranks' nnz)."""
    rows = int(bounds[-1])
    total = int(offsets[-1])
    rp = np.zeros(rows + 1, np.int64)
    ci = np.zeros(total, np.int32)
    va = np.zeros(total, np.float64)
    for r, blk in enumerate(blocks):
        r0, r1 = int(bounds[r]), int(bounds[r + 1])
        e0, e1 = int(offsets[r]), int(offsets[r + 1])
        if blk.rows != r1 - r0 or blk.nnz != e1 - e0:
            raise ValueError(f"block {r} does not match its bounds / offsets")
        rp[r0:r1 + 1] = global_row_ptr(blk.row_ptr, e0)
        ci[e0:e1] = blk.col_idx
        va[e0:e1] = blk.val
    return Csr(rows, cols, rp, ci, va)


def _spec_in(spec) -> CsrIn:
    rows, cols, nnz, rp, ci, va = spec
    return CsrIn(int(rows), int(cols), int(nnz), rp, ci, va)


class Communicator:
    """One rank of a multi-GPU product (one process per GPU)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = ct.create_string_buffer(ID_BYTES)
        _check(load().appt_comm_unique_id(buf), "appt_comm_unique_id")
        return buf.raw

    def __init__(self, uid: bytes, nranks: int, rank: int, device: int):
        if len(uid) != ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        self.nranks, self.rank, self.device = int(nranks), int(rank), int(device)
        self._h = ct.c_void_p()
        idb = ct.create_string_buffer(uid, ID_BYTES)
        _check(load().appt_comm_init(idb, self.nranks, self.rank, self.device,
                                     ct.byref(self._h)), "appt_comm_init")

    def destroy(self) -> None:
        if self._h:
            load().appt_comm_destroy(self._h)
            self._h = ct.c_void_p()

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    def broadcast_csr(self, root: int, spec=None):
        """Replicate a device CSR (rows, cols, nnz, row_ptr, col_idx, val) held by `root`.
        Returns (spec on this rank, transfer ms, owned): `owned` specs were allocated by the
        library (release them with free_csr)."""
        m = _spec_in(spec) if spec is not None else CsrIn()
        ms = ct.c_double(0.0)
        _check(load().appt_comm_broadcast_csr(self._h, int(root), ct.byref(m), ct.byref(ms)),
               "appt_comm_broadcast_csr")
        out = (int(m.rows), int(m.cols), int(m.nnz), m.row_ptr, m.col_idx, m.val)
        return out, float(ms.value), self.rank != root

    def free_csr(self, spec) -> None:
        m = _spec_in(spec)
        load().appt_comm_free_csr(self._h, ct.byref(m))

    def row_split(self, root: int, A_spec=None, B_spec=None) -> list[int]:
        """Row bounds of the ranks (nranks + 1), computed on the root from device-resident A
        (and B; B = A when None) and broadcast."""
        a = _spec_in(A_spec) if A_spec is not None else None
        b = _spec_in(B_spec) if B_spec is not None else None
        out = np.zeros(self.nranks + 1, np.int64)
        _check(load().appt_comm_row_split(self._h, int(root), ct.byref(a) if a else None,
                                          ct.byref(b) if b else None, out.ctypes.data),
               "appt_comm_row_split")
        return [int(x) for x in out]

    def multiply(self, A_block_spec, B_spec, op: str = "ab", row_base: int = 0,
                 method: str = "adaptive", stream=None, timing: bool = False) -> "CommMultiply":
        """A reusable call of this rank's block product on device-resident operands (see
        CommMultiply)."""
        return CommMultiply(self, A_block_spec, B_spec, op, row_base, method, stream, timing)

    def spgemm(self, A_block, B_spec, op: str = "ab", row_base: int = 0, out: str = "device",
               method: str = "adaptive", stream=None, timing: bool = False, copy: bool = True):
        """This rank's block of C. A_block: a host Csr, or a device spec tuple; B_spec: device
        spec of the replicated B. Returns (result, block_offsets): result is a DeviceResult
        (out="device") or a host Csr (out="host"; copy=False gives views of the library's
        pinned block)."""
        keep: list = []
        if isinstance(A_block, Csr):
            rp = np.ascontiguousarray(A_block.row_ptr, dtype=np.int32)
            ci = np.ascontiguousarray(A_block.col_idx, dtype=np.int32)
            va = np.ascontiguousarray(A_block.val, dtype=np.float64)
            keep += [rp, ci, va]
            a = CsrIn(A_block.rows, A_block.cols, int(rp[-1] - rp[0]), rp.ctypes.data,
                      ci.ctypes.data, va.ctypes.data)
            in_mem = MEM_HOST
        else:
            a = _spec_in(A_block)
            in_mem = MEM_DEVICE
        b = _spec_in(B_spec)
        o = _options(op, method, in_mem, MEM_HOST if out == "host" else MEM_DEVICE, row_base,
                     stream, self.device, timing, b_mem=B_DEVICE)
        res = CsrOut()
        st = Stats()
        offs = np.zeros(self.nranks + 1, np.int64)
        _check(load().appt_comm_spgemm(self._h, ct.byref(a), ct.byref(b), ct.byref(o),
                                       ct.byref(res), offs.ctypes.data, ct.byref(st)),
               "appt_comm_spgemm")
        if out == "host":
            if not copy:
                return _view_host_out(res), offs
            try:
                return _take_host_out(res), offs
            finally:
                load().appt_free_out(ct.byref(res))
        return DeviceResult(res, st), offs


class CommMultiply:
    """This rank's block of C = op(A, B) on device-resident operands with its call arguments built
    once: each run() makes one appt_comm_spgemm call (collective), releases the previous run's C
    block first, and leaves the block's device C and the ranks' offsets in .nnz / .offsets."""

    def __init__(self, comm: Communicator, A_block_spec, B_spec, op, row_base, method, stream,
                 timing):
        self._comm = comm
        self._lib = load()
        self._a = _spec_in(A_block_spec)
        self._b = _spec_in(B_spec)
        self._o = _options(op, method, MEM_DEVICE, MEM_DEVICE, row_base, stream, comm.device,
                           timing, b_mem=B_DEVICE)
        self._out = CsrOut()
        self._st = Stats()
        self.offsets = np.zeros(comm.nranks + 1, np.int64)
        self._live = False
        self.nnz = 0

    def run(self) -> "CommMultiply":
        self.free()
        _check(self._lib.appt_comm_spgemm(self._comm._h, ct.byref(self._a), ct.byref(self._b),
                                          ct.byref(self._o), ct.byref(self._out),
                                          self.offsets.ctypes.data, ct.byref(self._st)),
               "appt_comm_spgemm")
        self._live = True
        self.nnz = int(self._out.nnz)
        return self

    def phase_ms(self, phase: str) -> float:
        from . import PHASES
        return float(self._st.ms_phase[PHASES.index(phase)])

    @property
    def stats(self) -> dict:
        return self._st.as_dict()

    def free(self) -> None:
        if self._live:
            self._lib.appt_free_out(ct.byref(self._out))
            self._live = False

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
