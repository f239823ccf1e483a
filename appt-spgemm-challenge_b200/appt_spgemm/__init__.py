"""Python binding (ctypes) of libappt_spgemm.so, the B200 adaptive SpGEMM engine.

The engine is C++/CUDA behind the C ABI of include/appt_spgemm.h; this module only marshals
numpy arrays (host) or raw device pointers. It never computes a product itself: if the shared
library is missing, every call raises.

Two call styles mirror the library's two layers:

* reference-compatible: ``reference_entry("spgemm_self_product_adaptive", A)`` packs A into the
  reference's single host buffer layout and calls the exported entry point with the reference's
  signature (include/spgemm.h of XUE77565/APPT-Spgemm-Challenge), returning C parsed from the
  reference's output layout;
* native: ``spgemm(A, B=None, op="ab"|"aat"|"aat_upper", method=...)`` with int64 results and
  statistics, plus ``spgemm_device`` for operands already resident on the GPU.
"""
from __future__ import annotations

import ctypes as ct
import os
from pathlib import Path

import numpy as np

from .matrices import Csr

PKG_DIR = Path(__file__).resolve().parent.parent
# APPT_LIB selects another build of the library (e.g. a variant built with build.py)
LIB_PATH = Path(os.environ["APPT_LIB"]) if os.environ.get("APPT_LIB") else \
    PKG_DIR / "libappt_spgemm.so"

OPS = {"ab": 0, "aat": 1, "aat_upper": 2, "ab_upper": 3}
METHODS = {"adaptive": 0, "hash": 1, "merge": 2, "esc": 3}
MEM_HOST, MEM_DEVICE = 0, 1
NUM_BINS = 32
# Numeric tiers in bin order; the rank tiers come in three walks each (1, 2 or 4 lane groups
# per warp, chosen by the average length of the row's B rows).
BIN_NAMES = ["rank2k_g1", "rank2k_g2", "rank2k_g4", "rank4k_g1", "rank4k_g2", "rank4k_g4",
             "rank8k_g1", "rank8k_g2", "rank8k_g4", "hash64", "hash128", "hash256", "hash512",
             "hash1024", "hash_block", "window", "block_rank", "merge"]
PHASES = ["h2d", "transpose", "analyze", "symbolic", "scan", "numeric", "d2h", "other"]

# Reference entry points exported with C linkage (include/appt_spgemm.h, layer 1).
REFERENCE_ENTRIES = {
    "spgemm_self_product_adaptive": ("ab", False),
    "spgemm_self_product_hash": ("ab", False),
    "spgemm_self_product_merge3": ("ab", False),
    "spgemm_self_product_manual": ("ab", False),
    "spgemm_att_hash": ("aat_upper", True),
    "spgemm_att_merge3": ("aat_upper", True),
    "spgemm_att_adaptive": ("aat_upper", True),
    "spgemm_transpose_product": ("aat", False),
}


class CsrIn(ct.Structure):
    _fields_ = [("rows", ct.c_int64), ("cols", ct.c_int64), ("nnz", ct.c_int64),
                ("row_ptr", ct.c_void_p), ("col_idx", ct.c_void_p), ("val", ct.c_void_p)]


class CsrOut(ct.Structure):
    _fields_ = [("rows", ct.c_int64), ("cols", ct.c_int64), ("nnz", ct.c_int64),
                ("row_ptr", ct.c_void_p), ("col_idx", ct.c_void_p), ("val", ct.c_void_p),
                ("mem", ct.c_int32), ("device", ct.c_int32), ("opaque", ct.c_void_p)]


def _tier_rows(bin_rows) -> dict:
    """Rows per tier, the lane-group variants of a tier summed (rank2k_g1 + _g2 + _g4 -> rank2k)."""
    out: dict = {}
    for i, name in enumerate(BIN_NAMES):
        tier = name.split("_g")[0]
        out[tier] = out.get(tier, 0) + int(bin_rows[i])
    return out


class Stats(ct.Structure):
    _fields_ = [("products", ct.c_int64), ("c_nnz", ct.c_int64),
                ("bin_rows", ct.c_int64 * NUM_BINS), ("ms_total", ct.c_double),
                ("ms_phase", ct.c_double * 8), ("kernel_launches", ct.c_int64),
                ("method_used", ct.c_int32), ("pad", ct.c_int32)]

    def as_dict(self) -> dict:
        return {
            "products": int(self.products),
            "c_nnz": int(self.c_nnz),
            "bin_rows": {BIN_NAMES[i]: int(self.bin_rows[i]) for i in range(len(BIN_NAMES))},
            "tier_rows": _tier_rows(self.bin_rows),
            "ms_total": float(self.ms_total),
            "ms_phase": {PHASES[i]: float(self.ms_phase[i]) for i in range(8)},
            "kernel_launches": int(self.kernel_launches),
            "method_used": int(self.method_used),
        }


class Options(ct.Structure):
    _fields_ = [("op", ct.c_int32), ("method", ct.c_int32), ("in_mem", ct.c_int32),
                ("out_mem", ct.c_int32), ("row_base", ct.c_int64), ("stream", ct.c_void_p),
                ("device", ct.c_int32), ("timing", ct.c_int32), ("b_mem", ct.c_int32),
                ("reserved", ct.c_int32)]


class ApptError(RuntimeError):
    pass


_lib = None


def library_path() -> Path:
    return LIB_PATH


def load() -> ct.CDLL:
    """Load the in-tree shared library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ApptError(f"{LIB_PATH} not found: build it with appt-spgemm-challenge_b200/build.py")
    lib = ct.CDLL(str(LIB_PATH))
    lib.appt_spgemm.argtypes = [ct.POINTER(CsrIn), ct.POINTER(CsrIn), ct.POINTER(Options),
                                ct.POINTER(CsrOut), ct.POINTER(Stats)]
    lib.appt_spgemm.restype = ct.c_int
    lib.appt_free_out.argtypes = [ct.POINTER(CsrOut)]
    lib.appt_free_out.restype = ct.c_int
    lib.appt_transpose.argtypes = [ct.POINTER(CsrIn), ct.POINTER(Options), ct.POINTER(CsrOut)]
    lib.appt_transpose.restype = ct.c_int
    lib.appt_transpose_into.argtypes = [ct.POINTER(CsrIn), ct.POINTER(Options), ct.c_void_p,
                                        ct.c_void_p, ct.c_void_p]
    lib.appt_transpose_into.restype = ct.c_int
    lib.appt_row_products.argtypes = [ct.POINTER(CsrIn), ct.POINTER(CsrIn), ct.POINTER(Options),
                                      ct.c_void_p]
    lib.appt_row_products.restype = ct.c_int
    lib.appt_estimate_row_nnz.argtypes = [ct.POINTER(CsrIn), ct.c_int32, ct.POINTER(Options),
                                          ct.c_void_p]
    lib.appt_estimate_row_nnz.restype = ct.c_int
    lib.appt_estimate_row_nnz_with.argtypes = [ct.POINTER(CsrIn), ct.c_int32, ct.c_int32,
                                               ct.POINTER(Options), ct.c_void_p]
    lib.appt_estimate_row_nnz_with.restype = ct.c_int
    lib.appt_reference_score.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int64]
    lib.appt_reference_score.restype = ct.c_double
    lib.appt_last_error.restype = ct.c_char_p
    lib.appt_device_count.restype = ct.c_int
    lib.appt_release_cached.argtypes = [ct.c_int]
    lib.appt_release_cached.restype = ct.c_int
    lib.appt_kernel_launches.restype = ct.c_int64
    lib.appt_version.restype = ct.c_char_p
    lib.appt_default_options.argtypes = [ct.POINTER(Options)]
    sig = [ct.c_void_p, ct.c_int, ct.c_int, ct.c_int, ct.POINTER(ct.c_void_p),
           ct.POINTER(ct.c_int), ct.POINTER(ct.c_int), ct.POINTER(ct.c_int)]
    for name in REFERENCE_ENTRIES:
        fn = getattr(lib, name)
        fn.argtypes = sig
        fn.restype = None
    lib.mempool_init.argtypes = [ct.c_size_t]
    lib.mempool_init.restype = ct.c_bool
    lib.mempool_destroy.argtypes = []
    lib.pinned_free.argtypes = [ct.c_void_p]
    lib.pinned_d2h_alloc.argtypes = [ct.POINTER(ct.c_void_p), ct.c_size_t]
    lib.pinned_d2h_alloc.restype = ct.c_int
    lib.should_run_method.argtypes = [ct.c_char_p]
    lib.should_run_method.restype = ct.c_bool
    lib.build_csc.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_int,
                              ct.POINTER(ct.c_void_p), ct.POINTER(ct.c_void_p),
                              ct.POINTER(ct.c_void_p)]
    lib.build_csc.restype = None
    lib.mempool_cap.restype = ct.c_size_t
    vp, i64p = ct.c_void_p, ct.POINTER(ct.c_int64)
    lib.appt_split_rows.argtypes = [vp, ct.c_int64, ct.c_int, vp]
    lib.appt_split_rows.restype = ct.c_int
    lib.appt_comm_unique_id.argtypes = [vp]
    lib.appt_comm_unique_id.restype = ct.c_int
    lib.appt_comm_init.argtypes = [vp, ct.c_int, ct.c_int, ct.c_int, ct.POINTER(vp)]
    lib.appt_comm_init.restype = ct.c_int
    lib.appt_comm_destroy.argtypes = [vp]
    lib.appt_comm_destroy.restype = ct.c_int
    lib.appt_comm_broadcast_csr.argtypes = [vp, ct.c_int, ct.POINTER(CsrIn), ct.POINTER(ct.c_double)]
    lib.appt_comm_broadcast_csr.restype = ct.c_int
    lib.appt_comm_free_csr.argtypes = [vp, ct.POINTER(CsrIn)]
    lib.appt_comm_free_csr.restype = ct.c_int
    lib.appt_comm_row_split.argtypes = [vp, ct.c_int, ct.POINTER(CsrIn), ct.POINTER(CsrIn), vp]
    lib.appt_comm_row_split.restype = ct.c_int
    lib.appt_comm_spgemm.argtypes = [vp, ct.POINTER(CsrIn), ct.POINTER(CsrIn), ct.POINTER(Options),
                                     ct.POINTER(CsrOut), vp, ct.POINTER(Stats)]
    lib.appt_comm_spgemm.restype = ct.c_int
    del i64p
    lib.mempool_used.restype = ct.c_size_t
    _lib = lib
    return lib


def last_error() -> str:
    return load().appt_last_error().decode()


def device_count() -> int:
    return int(load().appt_device_count())


def release_cached(device: int = 0) -> None:
    """Return the library's cached pool memory on `device` to the driver."""
    _check(load().appt_release_cached(device), "appt_release_cached")


def kernel_launches() -> int:
    return int(load().appt_kernel_launches())


def version() -> str:
    return load().appt_version().decode()


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise ApptError(f"{what} failed (status {rc}): {last_error()}")


def _host_in(A: Csr, keep: list) -> CsrIn:
    rp = np.ascontiguousarray(A.row_ptr, dtype=np.int32)
    ci = np.ascontiguousarray(A.col_idx, dtype=np.int32)
    va = np.ascontiguousarray(A.val, dtype=np.float64)
    keep += [rp, ci, va]
    return CsrIn(A.rows, A.cols, int(rp[-1] - rp[0]), rp.ctypes.data, ci.ctypes.data,
                 va.ctypes.data)


B_AS_A, B_HOST, B_DEVICE = 0, 1, 2


def _options(op="ab", method="adaptive", in_mem=MEM_HOST, out_mem=MEM_HOST, row_base=0,
             stream=None, device=0, timing=False, b_mem=B_AS_A) -> Options:
    o = Options()
    o.b_mem = b_mem
    o.op = OPS[op] if isinstance(op, str) else int(op)
    o.method = METHODS[method] if isinstance(method, str) else int(method)
    o.in_mem, o.out_mem = in_mem, out_mem
    o.row_base = int(row_base)
    o.stream = stream
    o.device = device
    o.timing = 1 if timing else 0
    return o


def _take_host_out(out: CsrOut) -> Csr:
    rows, nnz = int(out.rows), int(out.nnz)
    rp = np.ctypeslib.as_array(ct.cast(out.row_ptr, ct.POINTER(ct.c_int64)), (rows + 1,)).copy()
    if nnz:
        ci = np.ctypeslib.as_array(ct.cast(out.col_idx, ct.POINTER(ct.c_int32)), (nnz,)).copy()
        va = np.ctypeslib.as_array(ct.cast(out.val, ct.POINTER(ct.c_double)), (nnz,)).copy()
    else:
        ci = np.zeros(0, np.int32)
        va = np.zeros(0, np.float64)
    return Csr(rows, int(out.cols), rp, ci, va)


class _HostOut:
    """Owner of a host result block (released to the library when the last view goes away)."""

    def __init__(self, out: CsrOut):
        self.out = out

    def __del__(self):
        try:
            load().appt_free_out(ct.byref(self.out))
        except Exception:
            pass


def _view_host_out(out: CsrOut) -> Csr:
    """Csr whose arrays are views of the library's (pinned) result block; the block is released
    when the Csr is (keep the Csr, not only its arrays)."""
    owner = _HostOut(out)
    rows, nnz = int(out.rows), int(out.nnz)

    def view(ptr, ctype, n, dtype):
        if n == 0:
            return np.zeros(0, dtype)
        return np.frombuffer((ctype * n).from_address(ptr), dtype=dtype)

    rp = np.frombuffer((ct.c_int64 * (rows + 1)).from_address(out.row_ptr), dtype=np.int64)
    ci = view(out.col_idx, ct.c_int32, nnz, np.int32)
    va = view(out.val, ct.c_double, nnz, np.float64)
    C = Csr(rows, int(out.cols), rp, ci, va)
    C._owner = owner
    return C


def spgemm(A: Csr, B: Csr | None = None, op: str = "ab", method: str = "adaptive",
           device: int = 0, timing: bool = False, return_stats: bool = False,
           copy: bool = True):
    """C = op(A, B) with host operands; returns a Csr with int64 row_ptr (and stats). With
    copy=False the arrays are views of the library's pinned result block (no host copy), valid
    while the returned Csr is alive."""
    lib = load()
    keep: list = []
    a = _host_in(A, keep)
    b = _host_in(B, keep) if B is not None else None
    o = _options(op, method, MEM_HOST, MEM_HOST, 0, None, device, timing)
    out = CsrOut()
    st = Stats()
    rc = lib.appt_spgemm(ct.byref(a), ct.byref(b) if b is not None else None, ct.byref(o),
                         ct.byref(out), ct.byref(st))
    _check(rc, "appt_spgemm")
    if not copy:
        C = _view_host_out(out)
        return (C, st.as_dict()) if return_stats else C
    try:
        C = _take_host_out(out)
    finally:
        lib.appt_free_out(ct.byref(out))
    return (C, st.as_dict()) if return_stats else C


class DeviceResult:
    """C returned in device memory (pool allocations owned by the library)."""

    def __init__(self, out: CsrOut, stats: Stats):
        self._out = out
        self._stats = stats
        self._stats_dict = None
        self.rows, self.cols, self.nnz = int(out.rows), int(out.cols), int(out.nnz)
        self.row_ptr, self.col_idx, self.val = out.row_ptr, out.col_idx, out.val

    @property
    def stats(self) -> dict:
        """The call's statistics as a dict (built on first access)."""
        if self._stats_dict is None:
            self._stats_dict = self._stats.as_dict()
        return self._stats_dict

    def phase_ms(self, phase: str) -> float:
        """Device time of one phase of the call (with timing=True), without building the dict."""
        return float(self._stats.ms_phase[PHASES.index(phase)])

    def free(self) -> None:
        if self._out is not None:
            load().appt_free_out(ct.byref(self._out))
            self._out = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def spgemm_device(rows: int, cols: int, nnz: int, row_ptr: int, col_idx: int, val: int,
                  B: tuple | None = None, op: str = "ab", method: str = "adaptive",
                  row_base: int = 0, stream: int | None = None, device: int = 0,
                  timing: bool = False) -> DeviceResult:
    """Operands given as raw device pointers (e.g. torch tensors' data_ptr()); C stays on the
    device. B, if given, is (rows, cols, nnz, row_ptr, col_idx, val)."""
    lib = load()
    a = CsrIn(rows, cols, nnz, row_ptr, col_idx, val)
    b = CsrIn(*B) if B is not None else None
    o = _options(op, method, MEM_DEVICE, MEM_DEVICE, row_base, stream, device, timing)
    out = CsrOut()
    st = Stats()
    rc = lib.appt_spgemm(ct.byref(a), ct.byref(b) if b is not None else None, ct.byref(o),
                         ct.byref(out), ct.byref(st))
    _check(rc, "appt_spgemm")
    return DeviceResult(out, st)


class DeviceMultiply:
    """Repeated C = op(A, B) on device-resident operands whose call arguments are built once:
    each run() makes one appt_spgemm call (C stays on the device, in the library's pool) and
    releases the previous run's C first. For loops that multiply the same resident operands
    again and again, where rebuilding the ctypes arguments would cost host time per call."""

    def __init__(self, rows: int, cols: int, nnz: int, row_ptr: int, col_idx: int, val: int,
                 B: tuple | None = None, op: str = "ab", method: str = "adaptive",
                 row_base: int = 0, stream: int | None = None, device: int = 0,
                 timing: bool = False):
        self._lib = load()
        self._a = CsrIn(rows, cols, nnz, row_ptr, col_idx, val)
        self._b = CsrIn(*B) if B is not None else None
        self._bref = ct.byref(self._b) if self._b is not None else None
        self._o = _options(op, method, MEM_DEVICE, MEM_DEVICE, row_base, stream, device, timing)
        self._out = CsrOut()
        self._st = Stats()
        self._live = False
        self.nnz = 0

    def run(self) -> "DeviceMultiply":
        self.free()
        _check(self._lib.appt_spgemm(ct.byref(self._a), self._bref, ct.byref(self._o),
                                     ct.byref(self._out), ct.byref(self._st)), "appt_spgemm")
        self._live = True
        self.nnz = int(self._out.nnz)
        return self

    def phase_ms(self, phase: str) -> float:
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


def transpose(A: Csr, device: int = 0) -> Csr:
    lib = load()
    keep: list = []
    a = _host_in(A, keep)
    o = _options("ab", "adaptive", MEM_HOST, MEM_HOST, 0, None, device)
    out = CsrOut()
    _check(lib.appt_transpose(ct.byref(a), ct.byref(o), ct.byref(out)), "appt_transpose")
    try:
        return _take_host_out(out)
    finally:
        lib.appt_free_out(ct.byref(out))


def transpose_into_device(rows: int, cols: int, nnz: int, row_ptr: int, col_idx: int, val: int,
                          t_row_ptr: int, t_col_idx: int, t_val: int, stream: int | None = None,
                          device: int = 0) -> None:
    """A^T of a device-resident A into caller-allocated device buffers (int32 row_ptr of
    cols + 1 entries, nnz column indices and values) -- the operand format, so it can be passed
    as B of spgemm_device."""
    lib = load()
    a = CsrIn(rows, cols, nnz, row_ptr, col_idx, val)
    o = _options("ab", "adaptive", MEM_DEVICE, MEM_DEVICE, 0, stream, device)
    _check(lib.appt_transpose_into(ct.byref(a), ct.byref(o), t_row_ptr, t_col_idx, t_val),
           "appt_transpose_into")


def row_products(A: Csr, B: Csr | None = None, device: int = 0) -> np.ndarray:
    lib = load()
    keep: list = []
    a = _host_in(A, keep)
    b = _host_in(B, keep) if B is not None else None
    o = _options(device=device)
    out = np.zeros(A.rows, dtype=np.int64)
    _check(lib.appt_row_products(ct.byref(a), ct.byref(b) if b is not None else None,
                                 ct.byref(o), out.ctypes.data), "appt_row_products")
    return out


ESTIMATORS = {"default": 0, "minhash": 1, "hll": 2}


def estimate_row_nnz(A: Csr, att: bool = False, device: int = 0,
                     estimator: str = "default") -> np.ndarray:
    """The reference's per-row output-size estimate; estimator "default" follows EST_METHOD
    like the reference, "minhash" or "hll" pick one explicitly."""
    lib = load()
    keep: list = []
    a = _host_in(A, keep)
    o = _options(device=device)
    out = np.zeros(A.rows, dtype=np.int32)
    _check(lib.appt_estimate_row_nnz_with(ct.byref(a), 1 if att else 0, ESTIMATORS[estimator],
                                          ct.byref(o), out.ctypes.data),
           "appt_estimate_row_nnz_with")
    return out


def reference_score(A: Csr) -> float:
    rp = np.ascontiguousarray(A.row_ptr, dtype=np.int32)
    return float(load().appt_reference_score(rp.ctypes.data, A.rows, A.nnz))


# ----------------------------------------------------------------------------- reference layout
def _align8(x: int) -> int:
    return (x + 7) & ~7


def pack_reference_buffer(A: Csr, out: np.ndarray | None = None) -> np.ndarray:
    """A in the reference's single host buffer layout: row_ptr | col_idx | pad8 | val
    (src/matrix_utils.cu:142-145). `out` may be a preallocated (e.g. pinned) uint8 array."""
    rp_b = 4 * (A.rows + 1)
    ci_b = 4 * A.nnz
    v_off = _align8(rp_b + ci_b)
    total = v_off + 8 * A.nnz
    buf = np.zeros(total, dtype=np.uint8) if out is None else out[:total]
    buf[:rp_b] = np.frombuffer(np.ascontiguousarray(A.row_ptr, np.int32).tobytes(), np.uint8)
    buf[rp_b:rp_b + ci_b] = np.frombuffer(np.ascontiguousarray(A.col_idx, np.int32).tobytes(),
                                          np.uint8)
    buf[v_off:v_off + 8 * A.nnz] = np.frombuffer(np.ascontiguousarray(A.val, np.float64).tobytes(),
                                                 np.uint8)
    return buf


def reference_buffer_bytes(A: Csr) -> int:
    return _align8(4 * (A.rows + 1) + 4 * A.nnz) + 8 * A.nnz


def unpack_reference_output(ptr: int, rows: int, cols: int, nnz: int) -> Csr:
    """Parse C from the reference's output layout row_ptr | pad8 | col_idx | pad8 | val
    (src/main.cu:185-193)."""
    rp_al = _align8(4 * (rows + 1))
    ci_al = _align8(4 * nnz)
    base = ptr
    rp = np.ctypeslib.as_array(ct.cast(base, ct.POINTER(ct.c_int32)), (rows + 1,)).copy()
    if nnz:
        ci = np.ctypeslib.as_array(ct.cast(base + rp_al, ct.POINTER(ct.c_int32)), (nnz,)).copy()
        va = np.ctypeslib.as_array(ct.cast(base + rp_al + ci_al, ct.POINTER(ct.c_double)),
                                   (nnz,)).copy()
    else:
        ci = np.zeros(0, np.int32)
        va = np.zeros(0, np.float64)
    return Csr(rows, cols, rp, ci, va)


def set_mempool(on: bool, dev_pool: bool = False, cap_bytes: int = 0) -> None:
    """Set the reference's USE_MEMPOOL / USE_DEV_POOL switches (g_use_mempool, g_use_dev_pool)
    and initialise the pinned arena, as the reference's main() does."""
    lib = load()
    ct.c_bool.in_dll(lib, "g_use_mempool").value = bool(on)
    ct.c_bool.in_dll(lib, "g_use_dev_pool").value = bool(dev_pool)
    if on and not lib.mempool_init(cap_bytes):
        raise ApptError(f"mempool_init failed: {last_error()}")


def reference_entry(name: str, A: Csr, buffer: np.ndarray | None = None,
                    parse: bool = True):
    """Call a reference-compatible entry point on host A. Returns (C, C_rows, C_cols, C_nnz);
    C is None when C_nnz < 0 (the reference's failure convention)."""
    lib = load()
    fn = getattr(lib, name)
    buf = pack_reference_buffer(A) if buffer is None else buffer
    cbuf = ct.c_void_p()
    cr, cc, cn = ct.c_int(), ct.c_int(), ct.c_int()
    fn(ct.c_void_p(buf.ctypes.data), A.rows, A.cols, A.nnz, ct.byref(cbuf), ct.byref(cr),
       ct.byref(cc), ct.byref(cn))
    if cn.value < 0 or not cbuf.value:
        return None, cr.value, cc.value, cn.value
    C = None
    if parse:
        true_cols = A.rows if REFERENCE_ENTRIES.get(name, ("ab",))[0] != "ab" else A.cols
        C = unpack_reference_output(cbuf.value, cr.value, true_cols, cn.value)
    lib.pinned_free(cbuf)
    return C, cr.value, cc.value, cn.value
