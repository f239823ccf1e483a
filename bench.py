#!/usr/bin/env python
"""Benchmark of the B200 adaptive SpGEMM engine.

Default workload (one GPU): C = A*A for the 27-point stencil on a 64^3 grid (n = 262,144,
fp64; seeded synthetic input standing in for the reference's SuiteSparse matrices).
Metric: GFLOPS = 2 x intermediate products / time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload stencil27|uniform8|rmat|banded|zipf_att]

A "step" is one full pass of the engine over the batch: analysis, symbolic count, scan,
numeric accumulation into a freshly allocated C (device pool), plus, with N > 1 GPUs, the
int64 nnz-offset all-gather. Rows of A are split across ranks by intermediate-product prefix;
B (or A^T) is replicated to every GPU with one NCCL broadcast before timing. The stencil
workload scales weakly (grid 64 x 64 x 64N); the others keep the matrix fixed (strong scaling).
zipf_att (C = A*A^T, ~817 GB dense-ish output) is computed in row blocks against a
device-resident A^T, each block released after it is formed.

`value` is device time (CUDA events on the launching stream, L2 flushed between steps, max over
ranks). `e2e` is the same metric through the reference-facing C entry point
(spgemm_self_product_adaptive / spgemm_transpose_product, pinned host buffers, N = 1) or the
native host-buffer appt_spgemm call per row block (N > 1), host<->device copies included; it is
null when C does not fit a host buffer.

--impl reference runs the reference's own adaptive CUDA build (oracle/_ref/ref_spgemm, the
unmodified reference sources) on the same workload through its host-buffer API on one GPU; when
that binary is absent it times the CPU oracle instead.
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


def _wl():
    from appt_spgemm import matrices as M
    return {
        "stencil27": {"name": "stencil27_64cube_AxA", "op": "ab", "weak": True,
                      "gen": lambda n: M.stencil27(64, gz=64 * n),
                      "data": "27-point stencil, values U(0.5,1.5), seed 1",
                      "dominant": "num_warp_rank_kernel"},
        "uniform8": {"name": "uniform8_n4096_AxA", "op": "ab", "weak": False,
                     "gen": lambda n: M.uniform8(), "data": "8 uniform cols/row, U(-1,1), seed 0",
                     "dominant": "num_warp_rank_kernel"},
        "rmat": {"name": "rmat_2^20_16M_AxA", "op": "ab", "weak": False,
                 "gen": lambda n: M.rmat(), "data": "R-MAT (.57,.19,.19,.05), U(0,1), seed 2",
                 "dominant": "num_block_rank_kernel"},
        "banded": {"name": "banded_2^22_w256_AxA", "op": "ab", "weak": False,
                   "gen": lambda n: M.banded(), "data": "16 cols/row within +-256, U(-1,1), seed 4",
                   "dominant": "num_warp_rank_kernel"},
        "zipf_att": {"name": "zipf_2^18x2^16_AxAT_streamed", "op": "aat", "weak": False,
                     "gen": lambda n: M.zipf_att(), "data": "Zipf(1.1) cols, U(-1,1), seed 3",
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
    return ap.parse_args()


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
    """SM clocks and throttle reasons during the timed region, polled through NVML every 2 ms
    (the timed regions are milliseconds long, too short for nvidia-smi's loop)."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
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

    def _run(self):
        nv = self.nv
        while not self.stop_flag.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                self.mask |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.002)

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


def clock_sampler(device: int):
    try:
        return NvmlClockSampler(device)
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


def traffic_from_profiles(tag: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    f = ROOT / "profiles" / f"{tag}.txt"
    if not f.exists():
        return None, None
    for ln in f.read_text().splitlines():
        if ln.startswith("traffic_bytes_per_launch:"):
            try:
                return float(ln.split(":", 1)[1].strip()), str(f.relative_to(ROOT))
            except ValueError:
                return None, None
    return None, None


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    wl = _wl()[args.workload]
    from appt_spgemm import matrices as M
    A = wl["gen"](1)
    ref_bin = ROOT / "oracle" / "_ref" / "ref_spgemm"
    line = {"metric": METRIC, "unit": UNIT, "higher_is_better": True, "impl": "reference",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "data": f"synthetic ({wl['data']})", "dtype": "f64",
            "scaling": "weak" if wl["weak"] else "strong", "vs_baseline": None,
            "config": {"workload": wl["name"], "rows": A.rows, "nnz_a": A.nnz}}
    if ref_bin.exists():
        method = "att_adaptive" if wl["op"] == "aat" else "adaptive"
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
            print(json.dumps({"impl": "reference", "metric": METRIC, "unit": UNIT,
                              "config": line["config"],
                              "unavailable": f"reference build on {wl['name']} {why}"}))
            return 0
        res = json.loads([ln for ln in r.stdout.splitlines()
                          if ln.startswith("{\"products\"")][-1])
        ms = float(np.mean(res["ms"]))
        val = 2.0 * res["products"] / (ms * 1e-3) / 1e9
        comp = reference_compute_only_ms(r.stderr, args.steps)
        line.update({"value": val, "ms_per_step": ms, "clocks": clocks,
                     "cpu_baseline": {"value": val, "unit": UNIT, "cores": 1, "kind": "reference",
                                      "sample": "full workload through the reference's own "
                                                f"{method} CUDA build (host-buffer API, one B200, "
                                                "one host thread); wall time per call"},
                     "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0},
                     "c_nnz": res["c_nnz"], "products": res["products"]})
        if comp is not None:
            line["compute_only"] = {
                "ms_per_call": comp, "value": 2.0 * res["products"] / (comp * 1e-3) / 1e9,
                "unit": UNIT,
                "rule": "the reference's own cudaEvent phase profile: TOTAL(GPU) - h2d - d2h, "
                        "mean over the timed calls"}
        line["config"]["reference"] = ("oracle/_ref/ref_spgemm (unmodified reference sources, "
                                       "sm_100a, USE_MEMPOOL=1)")
    else:
        cpu = cpu_baseline(A, wl["op"])
        line.update({"value": cpu["value"], "ms_per_step": cpu["ms"],
                     "cpu_baseline": cpu,
                     "e2e": {"value": cpu["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0}})
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


def cpu_baseline(A, op: str, budget_products: float = 4e10, min_seconds: float = 10.0):
    """CPU oracle (port) on a bounded row sample of the workload, all host threads; the sample is
    repeated until about `min_seconds` of CPU work have been timed."""
    import oracle
    from appt_spgemm import matrices as M
    from appt_spgemm.streaming import row_products_aat
    prods = row_products_aat(A) if op == "aat" else oracle.row_products(A)
    cum = np.cumsum(prods)
    r1 = int(np.searchsorted(cum, budget_products, side="right"))
    r1 = max(1, min(A.rows, r1))
    rp = np.asarray(A.row_ptr, np.int64)
    sub = M.Csr(r1, A.cols, (rp[:r1 + 1] - rp[0]).astype(np.int32), A.col_idx[:rp[r1]],
                A.val[:rp[r1]])
    B = oracle.transpose(A) if op == "aat" else A
    P = int(prods[:r1].sum())
    reps, dt = 0, 0.0
    while reps == 0 or dt < min_seconds:
        t0 = time.perf_counter()
        oracle.spgemm(sub, B, op="ab")
        dt += time.perf_counter() - t0
        reps += 1
    return {"value": 2.0 * P * reps / dt / 1e9, "unit": UNIT, "cores": oracle.num_threads(),
            "kind": "port", "ms": dt * 1e3 / reps,
            "sample": (f"first {r1} of {A.rows} rows ({P} products)" if r1 < A.rows
                       else f"full workload ({P} products)") +
                      f" x {reps} runs, {dt:.1f} s on the host cores"}


# ----------------------------------------------------------------------------- our arm
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
    from appt_spgemm import matrices as M
    from appt_spgemm.streaming import cut_blocks, row_products_aat

    wl = _wl()[args.workload]
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    # ---- workload on rank 0, replicated to every GPU with NCCL broadcasts
    if rank == 0:
        A = wl["gen"](world)
        sizes = torch.tensor([A.rows, A.cols, A.nnz], dtype=torch.int64, device=dev)
    else:
        A = None
        sizes = torch.zeros(3, dtype=torch.int64, device=dev)
    if world > 1:
        dist.broadcast(sizes, 0)
    rows, cols, nnz = (int(x) for x in sizes.tolist())
    if rank == 0:
        d_rp = torch.from_numpy(A.row_ptr).to(dev)
        d_ci = torch.from_numpy(A.col_idx).to(dev)
        d_va = torch.from_numpy(A.val).to(dev)
    else:
        d_rp = torch.empty(rows + 1, dtype=torch.int32, device=dev)
        d_ci = torch.empty(nnz, dtype=torch.int32, device=dev)
        d_va = torch.empty(nnz, dtype=torch.float64, device=dev)
    t_rep = 0.0
    if world > 1:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        D.replicate(dist, (d_rp, d_ci, d_va), 0)
        e1.record()
        torch.cuda.synchronize()
        t_rep = e0.elapsed_time(e1)
        if rank != 0:
            A = M.Csr(rows, cols, d_rp.cpu().numpy(), d_ci.cpu().numpy(), d_va.cpu().numpy())
    torch.cuda.synchronize()
    # a dedicated stream: the library's kernels, the L2 flush and the timing events share it
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream

    # ---- B operand: A itself, or A^T built on the device
    if wl["op"] == "aat":
        t_rp = torch.empty(cols + 1, dtype=torch.int32, device=dev)
        t_ci = torch.empty(nnz, dtype=torch.int32, device=dev)
        t_va = torch.empty(nnz, dtype=torch.float64, device=dev)
        ap.transpose_into_device(rows, cols, nnz, d_rp.data_ptr(), d_ci.data_ptr(),
                                 d_va.data_ptr(), t_rp.data_ptr(), t_ci.data_ptr(),
                                 t_va.data_ptr(), stream=sptr, device=local)
        Bspec = (cols, rows, nnz, t_rp.data_ptr(), t_ci.data_ptr(), t_va.data_ptr())
        B_rp_host = t_rp.cpu().numpy()
        prods = row_products_aat(A)
    else:
        Bspec = (rows, cols, nnz, d_rp.data_ptr(), d_ci.data_ptr(), d_va.data_ptr())
        B_rp_host = A.row_ptr
        prods = ap.row_products(A, device=local)

    # ---- rows of this rank (prefix-balanced), cut into blocks for streamed workloads
    bounds = D.partition_rows(prods, world)
    r0, r1 = bounds[rank], bounds[rank + 1]
    my_products = int(prods[r0:r1].sum())
    if wl["op"] == "aat":
        blocks = [r0 + b for b in cut_blocks(prods[r0:r1], args.block_products)]
    else:
        blocks = [r0, r1]
    rp_host = np.asarray(A.row_ptr, np.int64)

    def step():
        """One pass over this rank's rows; returns (nnz, numeric ms, the last block's result --
        its statistics are read after the timed region)."""
        nnz_tot, num_ms, st = 0, 0.0, None
        for b0, b1 in zip(blocks[:-1], blocks[1:]):
            res = ap.spgemm_device(b1 - b0, cols, int(rp_host[b1] - rp_host[b0]),
                                   d_rp.data_ptr() + 4 * b0, d_ci.data_ptr(), d_va.data_ptr(),
                                   B=Bspec, op="ab", method=args.method, row_base=b0,
                                   stream=sptr, device=local, timing=True)
            nnz_tot += res.nnz
            num_ms += res.phase_ms("numeric")
            st = res
            res.free()
        if world > 1:   # global row offsets of C: one all-gather, read on the host later
            D.exchange_nnz_into(dist, nnz_tot, nnz_all)
        return nnz_tot, num_ms, st

    nnz_all = torch.zeros(world, dtype=torch.int64, device=dev)

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    clk = clock_sampler(local)
    clk.start()
    launches0 = ap.kernel_launches()
    step_ms, num_ms = [], []
    c_nnz, stats = 0, None
    for _ in range(args.steps):
        flush.fill_(1)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        c_nnz, nms, stats = step()
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
    if world > 1:
        tt = torch.tensor([t_total, t_num], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_total_max = float(tt[0])
        pr = torch.tensor([my_products, c_nnz], dtype=torch.int64, device=dev)
        dist.all_reduce(pr)
        all_products, all_cnnz = int(pr[0]), int(pr[1])
        offs = D.block_offsets(nnz_all.cpu().numpy())   # the step's exchange, read once here
        if int(offs[-1]) != all_cnnz:
            raise RuntimeError(f"nnz exchange gave {int(offs[-1])} entries, ranks hold {all_cnnz}")
    else:
        t_total_max = t_total
        all_products, all_cnnz = my_products, c_nnz
    value = 2.0 * all_products * args.steps / (t_total_max * 1e-3) / 1e9

    peaks = measured_peaks()
    cbytes = compulsory_bytes(A, B_rp_host, r0, r1, c_nnz)
    achieved = cbytes / (t_num * 1e-3) / 1e9
    tr, tr_src = traffic_from_profiles(f"numeric_{args.workload}")

    e2e = None
    e2e_note = None
    c_bytes = 12 * c_nnz + 8 * (r1 - r0 + 1)
    if args.no_e2e:
        e2e_note = "skipped (--no-e2e)"
    elif c_bytes > E2E_MAX_C_BYTES or wl["op"] == "aat" and world > 1:
        e2e_note = f"C of this rank is {c_bytes / 2**30:.1f} GiB: not returned to a host buffer"
    else:
        e2e = e2e_measure(args, A, wl, r0, r1, world, rank, local, dist, torch)

    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(A, wl["op"])
        cpu.pop("ms", None)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_total_max / args.steps,
            "higher_is_better": True, "scaling": "weak" if wl["weak"] else "strong",
            "vs_baseline": None, "dtype": "f64", "data": f"synthetic ({wl['data']})",
            "config": {"workload": wl["name"] if world == 1 or not wl["weak"]
                       else f"stencil27_64x64x{64 * world}_AxA",
                       "rows": rows, "cols": cols, "nnz_a": nnz, "nnz_c": all_cnnz,
                       "products": all_products, "method": args.method,
                       "parallelism": f"row-sharded x{world}", "row_blocks": len(blocks) - 1,
                       "l2": "flushed between steps (256 MB write)",
                       "b_replication_ms": t_rep},
            "effective_gbs": cbytes / (t_total_max / args.steps * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": tr,
                         "kernel": f"numeric phase (dominant: {wl['dominant']})",
                         "algorithmic_bytes": cbytes, "avg_ms": t_num,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)"
                         if peaks["source"] == "measured" else "fallback 6.65 TB/s",
                         "traffic_source": tr_src},
            "phase_ms": stats.stats["ms_phase"] if stats else None,
            "bin_rows": ({k: v for k, v in stats.stats["bin_rows"].items() if v}
                         if stats else None),
            "clocks": clocks, "gpu_launches": launches,
            "e2e": e2e, "cpu_baseline": cpu,
        }
        if e2e_note:
            line["e2e_note"] = e2e_note
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def e2e_measure(args, A, wl, r0, r1, world, rank, local, dist, torch):
    import appt_spgemm as ap
    from appt_spgemm.streaming import row_products_aat
    if world == 1:
        ap.set_mempool(True, cap_bytes=0)
        nbytes = ap.reference_buffer_bytes(A)
        pinned = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        buf = ap.pack_reference_buffer(A, out=pinned.numpy())
        entry = "spgemm_transpose_product" if wl["op"] == "aat" else "spgemm_self_product_adaptive"
        times = []
        cn = 0
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
        P = int(row_products_aat(A).sum()) if wl["op"] == "aat" else \
            int(np.sum(ap.row_products(A, device=local)))
        d2h = ((4 * (A.rows + 1) + 7) & ~7) + ((4 * cn + 7) & ~7) + 8 * cn
        return {"value": 2.0 * P / t / 1e9, "unit": UNIT, "h2d_bytes_per_step": int(nbytes),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": t * 1e3,
                "api": f"{entry} (reference signature, pinned host buffers)"}
    def pinned(arr):
        src = torch.from_numpy(np.ascontiguousarray(arr))
        return torch.empty(src.shape, dtype=src.dtype, pin_memory=True).copy_(src).numpy()

    Ap = A.__class__(A.rows, A.cols, pinned(A.row_ptr), pinned(A.col_idx), pinned(A.val))
    blk = A.__class__(r1 - r0, A.cols, Ap.row_ptr[r0:r1 + 1], Ap.col_idx, Ap.val)
    times = []
    cnnz = 0
    for it in range(args.warmup + args.steps):
        dist.barrier()
        t0 = time.perf_counter()
        C = ap.spgemm(blk, Ap, op="ab", device=local, copy=False)   # C lands in pinned memory
        t1 = time.perf_counter()
        cnnz = C.nnz
        del C
        if it >= args.warmup:
            times.append(t1 - t0)
    dev = torch.device("cuda", local)
    t = torch.tensor([float(np.mean(times))], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    prods = torch.tensor([int(np.sum(ap.row_products(blk, A, device=local)))], dtype=torch.int64,
                         device=dev)
    dist.all_reduce(prods)
    h2d = 4 * (blk.rows + 1) + 12 * blk.nnz + 4 * (A.rows + 1) + 12 * A.nnz
    return {"value": 2.0 * int(prods[0]) / float(t[0]) / 1e9, "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(8 * (blk.rows + 1) + 12 * cnnz),
            "ms_per_step": float(t[0]) * 1e3,
            "api": "appt_spgemm (pinned host buffers in and out, row block of this rank)"}


if __name__ == "__main__":
    sys.exit(main())
