#!/usr/bin/env python
"""Benchmark of the B200 adaptive SpGEMM engine.

Default workload: C = A*A for the 27-point stencil on a 64^3 grid (n = 262,144, fp64; seeded
synthetic input standing in for the reference's SuiteSparse matrices). The matrix is fixed for
every GPU count (strong scaling): with N GPUs each rank computes a contiguous block of rows.
Metric: GFLOPS = 2 x intermediate products / time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload stencil27|uniform8|rmat|banded|zipf_att]

A "step" is one full pass of the engine over this rank's rows: analysis, symbolic count, scan,
numeric accumulation into a freshly allocated C (device pool) and, with N > 1 GPUs, the int64
nnz all-gather that places every rank's block in the global C (posted from inside the pipeline
and overlapped with the numeric phase). Multi-GPU runs use the library's own NCCL communicator
(appt_comm_*): B (or A^T) is replicated to every GPU with NCCL broadcasts before timing (its
device time is reported as b_replication_ms), rows are split by intermediate-product prefix.
zipf_att (C = A*A^T, about 825 GB of output) is computed in row blocks against a device-resident
A^T, each block released after it is formed (the same number of blocks on every rank).

`value` is device time (CUDA events on the launching stream, L2 flushed between steps, max over
ranks). `e2e` is the same metric through the public host-buffer entry points, copies included:
spgemm_self_product_adaptive (the reference's signature, pinned host buffers) at N = 1, and
appt_comm_spgemm with this rank's A block in pinned host memory, B resident on the device and
the C block returned to pinned host memory at N > 1 (max over ranks of the wall time).

--impl reference runs the reference's own adaptive CUDA build (oracle/_ref/ref_spgemm, built from
the unmodified reference sources) on the same workload on one GPU: `value` is its compute-only
time per call (its own phase profile, TOTAL(GPU) - h2d - d2h, the rule of the reference's
scripts/compare_methods.py), `e2e` its wall time per call through its host-buffer API.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "appt-spgemm-challenge_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "SpGEMM GFLOPS (2 x intermediate products / s)"
UNIT = "GFLOPS"
L2_FLUSH_BYTES = 256 << 20
E2E_MAX_C_BYTES = 16 << 30
STREAM_BLOCK_PRODUCTS = 1 << 32   # row blocks of streamed workloads: C <= 12 B x this, 48 GiB
INT32_MAX = (1 << 31) - 1


# Reduced instances for ncu captures (--size profile): the same generators, a few GB on the
# device at most, inputs or outputs still larger than L2.
PROFILE_SIZES = {"stencil27": {"g": 48}, "uniform8": {}, "rmat": {"scale": 16},
                 "banded": {"n": 1 << 20}, "zipf_att": {"rows": 1 << 14, "cols": 1 << 12}}


def _wl(size: str = "full"):
    from appt_spgemm import matrices as M
    if size == "profile":
        gens = {"stencil27": M.stencil27, "uniform8": M.uniform8, "rmat": M.rmat,
                "banded": M.banded, "zipf_att": M.zipf_att}
        out = _wl("full")
        for k, w in out.items():
            kw = PROFILE_SIZES[k]
            w["gen"] = (lambda g=gens[k], kw=kw: g(**kw))
            w["name"] = w["name"] + "_profile" + "".join(f"_{a}{b}" for a, b in kw.items())
            if kw:
                w["data"] += ", reduced: " + ", ".join(f"{a}={b}" for a, b in kw.items())
        return out
    return {
        "stencil27": {"name": "stencil27_64cube_AxA", "op": "ab",
                      "gen": lambda: M.stencil27(64),
                      "data": "27-point stencil 64^3, values U(0.5,1.5), seed 1",
                      "dominant": "num_warp_rank_kernel"},
        "uniform8": {"name": "uniform8_n4096_AxA", "op": "ab",
                     "gen": lambda: M.uniform8(), "data": "8 uniform cols/row, U(-1,1), seed 0",
                     "dominant": "num_warp_rank_kernel"},
        "rmat": {"name": "rmat_2^20_16M_AxA", "op": "ab",
                 "gen": lambda: M.rmat(), "data": "R-MAT (.57,.19,.19,.05), U(0,1), seed 2",
                 "dominant": "num_block_rank_kernel"},
        "banded": {"name": "banded_2^22_w256_AxA", "op": "ab",
                   "gen": lambda: M.banded(), "data": "16 cols/row within +-256, U(-1,1), seed 4",
                   "dominant": "num_warp_rank_kernel"},
        "zipf_att": {"name": "zipf_2^18x2^16_AxAT_streamed", "op": "aat",
                     "gen": lambda: M.zipf_att(), "data": "Zipf(1.1) cols, U(-1,1), seed 3",
                     "dominant": "num_block_window_kernel"},
    }


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="stencil27",
                    choices=["stencil27", "uniform8", "rmat", "banded", "zipf_att"])
    ap.add_argument("--method", default="adaptive")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--block-products", type=int, default=STREAM_BLOCK_PRODUCTS,
                    help="products per row block of the streamed A*A^T workload")
    ap.add_argument("--size", choices=["full", "profile"], default="full",
                    help="profile: reduced instances for ncu captures (not a benchmark line)")
    ap.add_argument("--clock-poll-ms", type=float, default=2.0,
                    help="NVML clock sampling interval during the timed region")
    ap.add_argument("--bind-cpus", choices=["off", "gpu"], default="off",
                    help="gpu: run each rank on the CPUs NVML reports as local to its GPU")
    return ap.parse_args()


def bind_to_gpu_cpus(device: int):
    """Restrict this process to the CPU cores NVML reports as nearest to `device` (its NUMA
    node); returns the number of cores, or None when NVML cannot tell."""
    try:
        import pynvml
        import torch
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        n = (os.cpu_count() + 63) // 64
        words = pynvml.nvmlDeviceGetCpuAffinity(h, n)
        cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:
        return None


def config_of(wl, A, c_nnz, products, method, world) -> dict:
    """The `config` object both arms print: the same keys and, for the same workload on one GPU,
    the same values, so the lines compare like for like (how each arm was run is in top-level
    keys)."""
    return {"workload": wl["name"], "rows": A.rows, "cols": A.cols, "nnz_a": A.nnz,
            "nnz_c": int(c_nnz), "products": int(products), "method": method,
            "parallelism": f"row-sharded x{world}" if world > 1 else "one GPU"}


# ----------------------------------------------------------------------------- helpers
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def compulsory_bytes(A, B_rp, r0: int, r1: int, c_nnz: int) -> int:
    """A block [4(m+1) + 12 nnz] + touched rows of B [12 len + 8 each] + C [8(m+1) + 12 nnz]."""
    rp = np.asarray(A.row_ptr, np.int64)
    brp = np.asarray(B_rp, np.int64)
    lo, hi = int(rp[r0]), int(rp[r1])
    m = r1 - r0
    a = 4 * (m + 1) + 12 * (hi - lo)
    ks = np.unique(A.col_idx[lo:hi])
    blen = brp[ks + 1] - brp[ks]
    b = int(12 * blen.sum() + 8 * ks.size)
    return a + b + 8 * (m + 1) + 12 * c_nnz


class NvmlClockSampler:
    """SM clocks and throttle reasons during the timed region, polled through NVML (every 2 ms by
    default, --clock-poll-ms; the timed regions are milliseconds long, too short for
    nvidia-smi's loop)."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int, poll_ms: float = 2.0):
        import pynvml
        import torch
        self.nv = pynvml
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        self.smax = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        self.sm: list[float] = []
        self.mask = 0
        self.stop_flag = threading.Event()
        self.thread = None
        self.poll_s = max(poll_ms, 0.1) * 1e-3

    def _run(self):
        nv = self.nv
        while not self.stop_flag.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                self.mask |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(self.poll_s)

    def start(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        self.stop_flag.set()
        self.thread.join(timeout=2)
        reasons = sorted(k for k, b in self.REASONS.items() if self.mask & b)
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None,
                "sm_max_mhz": float(self.smax), "reasons": reasons, "samples": len(self.sm),
                "source": "nvml"}


def clock_sampler(device: int, poll_ms: float = 2.0):
    try:
        return NvmlClockSampler(device, poll_ms)
    except Exception:
        return ClockSampler(device)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def traffic_from_profiles(tag: str, workload: str, rows: int):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary
    profiles/<tag>*.txt, used only when that summary names this very workload and row count (its
    "workload:" line reads "<name> rows=<rows>"; a summary captured on a smaller case of a uniform
    workload carries the traffic scaled to the full launch, and says so); else (None, None)."""
    want = f"workload: {workload} rows={rows}"
    for f in sorted((ROOT / "profiles").glob(f"{tag}*.txt")):
        lines = f.read_text().splitlines()
        if not any(ln.strip() == want for ln in lines):
            continue
        for ln in lines:
            if ln.startswith("traffic_bytes_per_launch:"):
                try:
                    return float(ln.split(":", 1)[1].strip()), str(f.relative_to(ROOT))
                except ValueError:
                    return None, None
    return None, None


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, rank: int, world: int):
    """The reference's own adaptive CUDA build on one GPU (rank 0 only)."""
    if rank != 0:
        return 0
    wl = _wl(args.size)[args.workload]
    from appt_spgemm import matrices as M
    A = wl["gen"]()
    ref_bin = ROOT / "oracle" / "_ref" / "ref_spgemm"
    method = "att_adaptive" if wl["op"] == "aat" else "adaptive"
    base = {"metric": METRIC, "unit": UNIT, "impl": "reference"}

    def unavailable(why: str) -> int:
        print(json.dumps({**base, "config": config_of(wl, A, 0, 0, args.method, 1),
                          "unavailable": why}), flush=True)
        return 0

    if not ref_bin.exists():
        return unavailable("oracle/_ref/ref_spgemm (the reference's CUDA build) is not built")
    if wl["op"] == "aat":
        return unavailable("the reference computes only the upper triangle of A*A^T, with int32 "
                           "counters that overflow on this workload (3.98e11 products)")
    prods = int(np.diff(np.asarray(A.row_ptr, np.int64))[A.col_idx].sum())
    if prods > INT32_MAX:
        return unavailable(f"the reference's int32 product and estimate counters overflow "
                           f"({prods} intermediate products)")
    if args.workload == "banded":
        # the reference sizes its hash temporaries from sum(est) in an int; on this matrix that sum
        # is 2,145,824,768 (0.077% under INT32_MAX, computed on the CPU by the oracle's
        # restatement of its MinHash estimate), too close to run it safely
        return unavailable("the reference's int32 sum of per-row estimates is 2,145,824,768 on "
                           "this matrix, 0.077% below INT32_MAX: not run")
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "a.bin"
        M.save_bin(path, A)
        clk = ClockSampler(0)
        clk.start()
        try:
            r = subprocess.run([str(ref_bin), method, str(path), "--warmup", str(args.warmup),
                                "--repeat", str(args.steps)], capture_output=True, text=True,
                               timeout=1200)
        except subprocess.TimeoutExpired:
            r = None
        clocks = clk.stop()
    if r is None or r.returncode != 0:
        why = "timed out" if r is None else \
            f"exited {r.returncode}: {' '.join(r.stderr.strip().splitlines()[-1:])[:200]}"
        return unavailable(f"reference build on {wl['name']} {why}")
    res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{\"products\"")][-1])
    wall = float(np.mean(res["ms"]))
    comp = reference_compute_only_ms(r.stderr, args.steps)
    P = int(res["products"])
    wall_val = 2.0 * P / (wall * 1e-3) / 1e9
    val, ms, rule = wall_val, wall, "wall time per call (no phase profile found)"
    if comp is not None:
        val = 2.0 * P / (comp * 1e-3) / 1e9
        ms = comp
        rule = ("compute only: the reference's own cudaEvent phase profile, TOTAL(GPU) - h2d - "
                "d2h per call (scripts/compare_methods.py:37-52), mean over the timed calls")
    cn = int(res["c_nnz"])
    h2d = ((4 * (A.rows + 1) + 4 * A.nnz + 7) & ~7) + 8 * A.nnz
    d2h = ((4 * (A.rows + 1) + 7) & ~7) + ((4 * cn + 7) & ~7) + 8 * cn
    line = {**base, "value": val, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": f"synthetic ({wl['data']})",
            "config": config_of(wl, A, cn, P, args.method, 1),
            "reference_build": "oracle/_ref/ref_spgemm (unmodified reference sources, sm_100a, "
                               "USE_MEMPOOL=1)",
            "value_rule": rule,
            "clocks": clocks,
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": 1, "kind": "reference",
                             "sample": f"full workload through the reference's own {method} "
                                       "CUDA build (one B200, one host thread)"},
            "e2e": {"value": wall_val, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": wall,
                    "api": f"spgemm_self_product_{method} of the reference (host buffers, "
                           "wall time per call)"},
            "gpu_launches": None}
    print(json.dumps(line), flush=True)
    return 0


def reference_compute_only_ms(stderr: str, calls: int):
    """Compute-only time per call from the reference's phase profiler lines
    ("[<tag>-prof] <phase> <ms>", one "TOTAL(GPU)" line per call): TOTAL - h2d - d2h."""
    import re
    pat = re.compile(r"\[(\w+)-prof\]\s+(\S.*?)\s+([0-9.]+) ms")
    per_call, cur = [], {}
    for ln in stderr.splitlines():
        m = pat.search(ln)
        if not m:
            continue
        name, ms = m.group(2).strip(), float(m.group(3))
        if name == "TOTAL(GPU)":
            per_call.append(ms - cur.get("h2d", 0.0) - cur.get("d2h", 0.0))
            cur = {}
        else:
            cur[name] = cur.get(name, 0.0) + ms
    if not per_call:
        return None
    tail = per_call[-calls:] if calls > 0 else per_call
    return float(np.mean(tail))


# ----------------------------------------------------------------------------- CPU baselines
def _row_sample(A, prods, budget_products):
    from appt_spgemm import matrices as M
    cum = np.cumsum(prods)
    r1 = int(np.searchsorted(cum, budget_products, side="right"))
    r1 = max(1, min(A.rows, r1))
    rp = np.asarray(A.row_ptr, np.int64)
    sub = M.Csr(r1, A.cols, (rp[:r1 + 1] - rp[0]).astype(np.int32), A.col_idx[:rp[r1]],
                A.val[:rp[r1]])
    return sub, r1, int(prods[:r1].sum())


def cpu_baseline(A, op: str, prods, budget_products: float = 4e10, min_seconds: float = 10.0):
    """The CPU oracle (a port of the reference's algorithm, OpenMP on all host threads) on a
    bounded row sample of the workload, repeated until about `min_seconds` are timed."""
    import oracle
    sub, r1, P = _row_sample(A, prods, budget_products)
    B = oracle.transpose(A) if op == "aat" else A
    reps, dt = 0, 0.0
    while reps == 0 or dt < min_seconds:
        t0 = time.perf_counter()
        oracle.spgemm(sub, B, op="ab")
        dt += time.perf_counter() - t0
        reps += 1
    return {"value": 2.0 * P * reps / dt / 1e9, "unit": UNIT, "cores": oracle.num_threads(),
            "kind": "port",
            "sample": (f"first {r1} of {A.rows} rows ({P} products)" if r1 < A.rows
                       else f"full workload ({P} products)") +
                      f" x {reps} runs, {dt:.1f} s on the host cores"}


def scipy_baseline(A, op: str, prods, budget_products: float = 2e9, min_seconds: float = 10.0):
    """scipy's CSR product (sparsetools, single-threaded) on a bounded row sample."""
    import scipy
    sub, r1, P = _row_sample(A, prods, budget_products)
    S = sub.to_scipy()
    B = A.to_scipy()
    B = B.T.tocsr() if op == "aat" else B
    reps, dt = 0, 0.0
    while reps == 0 or dt < min_seconds:
        t0 = time.perf_counter()
        C = S @ B
        dt += time.perf_counter() - t0
        reps += 1
        del C
    return {"value": 2.0 * P * reps / dt / 1e9, "unit": UNIT, "cores": 1,
            "host_cores": os.cpu_count(), "kind": "scipy", "version": scipy.__version__,
            "sample": (f"first {r1} of {A.rows} rows ({P} products)" if r1 < A.rows
                       else f"full workload ({P} products)") +
                      f" x {reps} runs, {dt:.1f} s, scipy.sparse csr @ csr (one thread)"}


# ----------------------------------------------------------------------------- our arm
class _CudaArray:
    """Zero-copy torch view of device memory the library owns (__cuda_array_interface__)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def _host_copy(torch, spec, local: int):
    """Host Csr of a device CSR spec (rows, cols, nnz, row_ptr, col_idx, val)."""
    from appt_spgemm import matrices as M
    rows, cols, nnz, rp, ci, va = spec
    d = f"cuda:{local}"
    trp = torch.as_tensor(_CudaArray(rp, rows + 1, "<i4"), device=d).cpu().numpy()
    tci = torch.as_tensor(_CudaArray(ci, max(nnz, 1), "<i4"), device=d)[:nnz].cpu().numpy()
    tva = torch.as_tensor(_CudaArray(va, max(nnz, 1), "<f8"), device=d)[:nnz].cpu().numpy()
    return M.Csr(rows, cols, trp, tci, tva)


def _pinned(torch, arr):
    src = torch.from_numpy(np.ascontiguousarray(arr))
    return torch.empty(src.shape, dtype=src.dtype, pin_memory=True).copy_(src).numpy()


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import appt_spgemm as ap
    from appt_spgemm import distributed as D
    from appt_spgemm.streaming import cut_blocks, row_products_aat

    wl = _wl(args.size)[args.workload]
    bound = bind_to_gpu_cpus(local) if args.bind_cpus == "gpu" else None
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:   # the harness's own group: id exchange, barriers, max over ranks
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    # ---- the matrix: generated on rank 0, replicated by the library's NCCL broadcast
    comm, t_rep, owned = None, 0.0, False
    tA, specA, A = None, None, None
    if rank == 0:
        A = wl["gen"]()
        tA = (torch.from_numpy(A.row_ptr).to(dev), torch.from_numpy(A.col_idx).to(dev),
              torch.from_numpy(A.val).to(dev))
        specA = (A.rows, A.cols, A.nnz, tA[0].data_ptr(), tA[1].data_ptr(), tA[2].data_ptr())
    if world > 1:
        ids = [D.Communicator.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        comm = D.Communicator(ids[0], world, rank, local)
        specA, t_rep, owned = comm.broadcast_csr(0, specA)
        if rank != 0:
            A = _host_copy(torch, specA, local)
    torch.cuda.synchronize()
    rows, cols, nnz = A.rows, A.cols, A.nnz
    # a dedicated stream: the library's kernels, the L2 flush and the timing events share it
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream

    # ---- B operand: A itself, or A^T built on the device
    if wl["op"] == "aat":
        t_rp = torch.empty(cols + 1, dtype=torch.int32, device=dev)
        t_ci = torch.empty(nnz, dtype=torch.int32, device=dev)
        t_va = torch.empty(nnz, dtype=torch.float64, device=dev)
        ap.transpose_into_device(rows, cols, nnz, specA[3], specA[4], specA[5], t_rp.data_ptr(),
                                 t_ci.data_ptr(), t_va.data_ptr(), stream=sptr, device=local)
        specB = (cols, rows, nnz, t_rp.data_ptr(), t_ci.data_ptr(), t_va.data_ptr())
        B_rp_host = t_rp.cpu().numpy()
        prods = row_products_aat(A)
    else:
        specB = specA
        B_rp_host = A.row_ptr
        prods = None

    # ---- rows of this rank (prefix-balanced products), blocks of streamed workloads
    if world > 1:
        bounds = comm.row_split(0, specA if rank == 0 else None,
                                specB if rank == 0 and wl["op"] == "aat" else None)
    else:
        bounds = [0, rows]
    r0, r1 = bounds[rank], bounds[rank + 1]
    if wl["op"] == "aat":   # the same number of blocks on every rank: the exchanges pair up
        K = max(len(cut_blocks(prods[bounds[r]:bounds[r + 1]], args.block_products)) - 1
                for r in range(world))
        blocks = [r0 + b for b in D.split_rows(prods[r0:r1], max(K, 1))]
    else:
        blocks = [r0, r1]
    rp_host = np.asarray(A.row_ptr, np.int64)

    def block_spec(b0, b1):
        return (b1 - b0, cols, int(rp_host[b1] - rp_host[b0]), specA[3] + 4 * b0, specA[4],
                specA[5])

    # one reusable call per row block: the arguments are built once, outside the timed region
    calls = []
    for b0, b1 in zip(blocks[:-1], blocks[1:]):
        if comm is None:
            calls.append(ap.DeviceMultiply(*block_spec(b0, b1), B=specB, op="ab",
                                           method=args.method, row_base=b0, stream=sptr,
                                           device=local, timing=True))
        else:
            calls.append(comm.multiply(block_spec(b0, b1), specB, op="ab", row_base=b0,
                                       method=args.method, stream=sptr, timing=True))

    def step():
        """One pass over this rank's rows: (nnz, numeric ms, last block's call -- its
        statistics are read after the timed region --, last exchange's offsets)."""
        nnz_tot, num_ms, st, offs = 0, 0.0, None, None
        for c in calls:
            c.run()
            nnz_tot += c.nnz
            num_ms += c.phase_ms("numeric")
            st = c
            offs = getattr(c, "offsets", None)
            c.free()
        return nnz_tot, num_ms, st, offs

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    clk = clock_sampler(local, args.clock_poll_ms)
    clk.start()
    launches0 = ap.kernel_launches()
    step_ms, num_ms = [], []
    c_nnz, stats, offs = 0, None, None
    for _ in range(args.steps):
        flush.fill_(1)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        c_nnz, nms, stats, offs = step()
        ev1.record(stream)
        ev1.synchronize()
        step_ms.append(ev0.elapsed_time(ev1))
        num_ms.append(nms)
    torch.cuda.synchronize()
    launches = ap.kernel_launches() - launches0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = clk.stop()

    t_total = float(sum(step_ms))
    t_num = float(np.mean(num_ms))
    my_products = int(stats.stats["products"]) if len(blocks) == 2 else \
        int(prods[r0:r1].sum())
    if world > 1:
        tt = torch.tensor([t_total, t_num], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_total_max = float(tt[0])
        pr = torch.tensor([my_products, c_nnz], dtype=torch.int64, device=dev)
        dist.all_reduce(pr)
        all_products, all_cnnz = int(pr[0]), int(pr[1])
        if len(blocks) == 2 and int(offs[-1]) != all_cnnz:
            raise RuntimeError(f"nnz exchange gave {int(offs[-1])} entries, ranks hold {all_cnnz}")
    else:
        t_total_max = t_total
        all_products, all_cnnz = my_products, c_nnz
    value = 2.0 * all_products * args.steps / (t_total_max * 1e-3) / 1e9

    peaks = measured_peaks()
    cbytes = compulsory_bytes(A, B_rp_host, r0, r1, c_nnz)
    achieved = cbytes / (t_num * 1e-3) / 1e9
    tr, tr_src = (traffic_from_profiles(f"numeric_{args.workload}", wl["name"], rows)
                  if world == 1 else (None, None))

    e2e, e2e_note = None, None
    c_bytes = 12 * c_nnz + 8 * (r1 - r0 + 1)
    if args.no_e2e:
        e2e_note = "skipped (--no-e2e)"
    elif c_bytes > E2E_MAX_C_BYTES or wl["op"] == "aat":
        e2e_note = f"C of this rank is {c_bytes / 2**30:.1f} GiB: not returned to a host buffer"
    elif world == 1:
        e2e = e2e_single(args, A, wl, local, torch)
    else:
        e2e = e2e_sharded(args, A, r0, r1, comm, specB, local, dist, torch)

    cpu, cpu_scipy = None, None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        import oracle
        p = prods if prods is not None else oracle.row_products(A)
        cpu = cpu_baseline(A, wl["op"], p)
        cpu_scipy = scipy_baseline(A, wl["op"], p)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_total_max / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": f"synthetic ({wl['data']})",
            "config": config_of(wl, A, all_cnnz, all_products, args.method, world),
            "l2": "flushed between steps (256 MB write)",
            "row_blocks_per_rank": len(blocks) - 1, "b_replication_ms": t_rep,
            "host": {"cpu_binding": f"GPU-local cores ({bound})" if bound else "none",
                     "clock_poll_ms": args.clock_poll_ms},
            "effective_gbs": cbytes / (t_total_max / args.steps * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": tr,
                         "kernel": f"numeric phase (dominant: {wl['dominant']})",
                         "algorithmic_bytes": cbytes, "avg_ms": t_num,
                         "rows_of_rank0": r1 - r0,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)"
                         if peaks["source"] == "measured" else "fallback 6.65 TB/s",
                         "traffic_source": tr_src},
            "phase_ms": stats.stats["ms_phase"] if stats else None,
            "bin_rows": ({k: v for k, v in stats.stats["bin_rows"].items() if v}
                         if stats else None),
            "clocks": clocks, "gpu_launches": launches,
            "e2e": e2e, "cpu_baseline": cpu, "cpu_baseline_scipy": cpu_scipy,
        }
        if e2e_note:
            line["e2e_note"] = e2e_note
        print(json.dumps(line), flush=True)
    if comm is not None:
        if owned:
            comm.free_csr(specA)
        comm.destroy()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def e2e_single(args, A, wl, local, torch):
    """One GPU, through the reference-signature entry point with pinned host buffers."""
    import appt_spgemm as ap
    ap.set_mempool(True, cap_bytes=0)
    nbytes = ap.reference_buffer_bytes(A)
    pinned = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    buf = ap.pack_reference_buffer(A, out=pinned.numpy())
    entry = "spgemm_self_product_adaptive"
    times, cn = [], 0
    for it in range(args.warmup + args.steps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _, _, _, cn = ap.reference_entry(entry, A, buffer=buf, parse=False)
        t1 = time.perf_counter()
        if cn < 0:
            raise RuntimeError(f"reference-facing entry failed: {ap.last_error()}")
        if it >= args.warmup:
            times.append(t1 - t0)
    t = float(np.mean(times))
    P = int(np.sum(ap.row_products(A, device=local)))
    d2h = ((4 * (A.rows + 1) + 7) & ~7) + ((4 * cn + 7) & ~7) + 8 * cn
    return {"value": 2.0 * P / t / 1e9, "unit": UNIT, "h2d_bytes_per_step": int(nbytes),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": t * 1e3,
            "api": f"{entry} (reference signature, pinned host buffers)"}


def e2e_sharded(args, A, r0, r1, comm, specB, local, dist, torch):
    """N GPUs: every rank's A block in pinned host memory goes in, its C block comes back to
    pinned host memory; B stays resident on every GPU (replicated once). Max over ranks."""
    from appt_spgemm import matrices as M
    rp = np.asarray(A.row_ptr, np.int64)
    e0, e1 = int(rp[r0]), int(rp[r1])
    blk = M.Csr(r1 - r0, A.cols, _pinned(torch, (rp[r0:r1 + 1] - e0).astype(np.int32)),
                _pinned(torch, A.col_idx[e0:e1]), _pinned(torch, A.val[e0:e1]))
    times, cnnz = [], 0
    for it in range(args.warmup + args.steps):
        dist.barrier()
        t0 = time.perf_counter()
        C, offs = comm.spgemm(blk, specB, op="ab", row_base=r0, out="host", copy=False)
        t1 = time.perf_counter()
        cnnz = C.nnz
        del C
        if it >= args.warmup:
            times.append(t1 - t0)
    dev = torch.device("cuda", local)
    t = torch.tensor([float(np.mean(times))], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    import appt_spgemm as ap
    pr = torch.tensor([int(np.sum(ap.row_products(blk, A, device=local)))], dtype=torch.int64,
                      device=dev)
    dist.all_reduce(pr)
    h2d = 4 * (blk.rows + 1) + 12 * blk.nnz
    return {"value": 2.0 * int(pr[0]) / float(t[0]) / 1e9, "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(8 * (blk.rows + 1) +
                                                                       12 * cnnz),
            "ms_per_step": float(t[0]) * 1e3,
            "api": "appt_comm_spgemm (this rank's A block from pinned host memory, B resident "
                   "on the GPU, C block to pinned host memory; max over ranks)"}


if __name__ == "__main__":
    sys.exit(main())
