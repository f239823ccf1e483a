#!/usr/bin/env python
"""Benchmark of the B200 adaptive SpGEMM engine.

Workload (one GPU): C = A*A for the 27-point stencil on a 64^3 grid (n = 262,144, fp64, seeded
synthetic input standing in for the reference's SuiteSparse matrices). Metric: GFLOPS =
2 x intermediate products / time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A "step" is one full pass of the engine over the batch: analysis, symbolic count, scan,
numeric accumulation into a freshly allocated C (device pool), plus, with N > 1 GPUs, the
int64 nnz-offset all-gather. With N GPUs the grid grows to 64 x 64 x (64 N) (weak scaling):
rank r computes a contiguous row block balanced by intermediate products, B = A is
replicated to every GPU with one NCCL broadcast before timing.

`value` is device time (CUDA events on the launching stream, L2 flushed between steps, max
over ranks); `e2e` is the same metric through the reference-facing C entry point
spgemm_self_product_adaptive with pinned host buffers (N = 1) or the native host-buffer
appt_spgemm call per row block (N > 1), host<->device copies included.

--impl reference runs the reference's own adaptive CUDA build (oracle/_ref/ref_spgemm,
unmodified reference sources) on the same workload through its host-buffer API on one GPU;
when that binary is absent it times the CPU oracle instead.
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
WORKLOAD = "stencil27_64cube_AxA"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--method", default="adaptive")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
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


def compulsory_bytes(A, r0: int, r1: int, c_nnz: int) -> int:
    """A block [4(m+1) + 12 nnz] + touched rows of B [12 len + 8 each] + C [8(m+1) + 12 nnz]."""
    rp = A.row_ptr.astype(np.int64)
    lo, hi = int(rp[r0]), int(rp[r1])
    m = r1 - r0
    a = 4 * (m + 1) + 12 * (hi - lo)
    ks = np.unique(A.col_idx[lo:hi])
    blen = (rp[ks + 1] - rp[ks])
    b = int(12 * blen.sum() + 8 * ks.size)
    c = 8 * (m + 1) + 12 * c_nnz
    return a + b + c


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


def traffic_from_profiles(kernel_tag: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary, if any."""
    f = ROOT / "profiles" / f"{kernel_tag}.txt"
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
    from appt_spgemm import matrices as M
    A = M.stencil27(64)
    ref_bin = ROOT / "oracle" / "_ref" / "ref_spgemm"
    line = {"metric": METRIC, "unit": UNIT, "higher_is_better": True, "impl": "reference",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "data": "synthetic",
            "dtype": "f64", "scaling": "weak", "vs_baseline": None,
            "config": {"workload": WORKLOAD, "rows": A.rows, "nnz_a": A.nnz}}
    if ref_bin.exists():
        with tempfile.TemporaryDirectory() as td:
            path = Path(td) / "a.bin"
            M.save_bin(path, A)
            clk = ClockSampler(0)
            clk.start()
            r = subprocess.run([str(ref_bin), "adaptive", str(path), "--warmup", str(args.warmup),
                                "--repeat", str(args.steps)], capture_output=True, text=True,
                               timeout=1200)
            clocks = clk.stop()
        if r.returncode != 0:
            print(json.dumps({"impl": "reference",
                              "unavailable": f"reference build exited {r.returncode}: "
                                             f"{r.stderr.strip().splitlines()[-1:]}"}))
            return 0
        res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{\"products\"")][-1])
        ms = float(np.mean(res["ms"]))
        val = 2.0 * res["products"] / (ms * 1e-3) / 1e9
        line.update({"value": val, "ms_per_step": ms, "clocks": clocks,
                     "cpu_baseline": {"value": val, "unit": UNIT, "cores": 1, "kind": "reference",
                                      "sample": "full workload through the reference's own "
                                                "adaptive CUDA build (host-buffer API, one B200, "
                                                "one host thread); wall time per call"},
                     "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0},
                     "c_nnz": res["c_nnz"], "products": res["products"]})
        line["config"]["reference"] = "oracle/_ref/ref_spgemm adaptive (unmodified reference " \
                                      "sources, sm_100a, USE_MEMPOOL=1)"
    else:
        import oracle
        t0 = time.perf_counter()
        C = oracle.spgemm(A)
        dt = time.perf_counter() - t0
        P = int(oracle.row_products(A).sum())
        val = 2.0 * P / dt / 1e9
        line.update({"value": val, "ms_per_step": dt * 1e3,
                     "cpu_baseline": {"value": val, "unit": UNIT, "cores": oracle.num_threads(),
                                      "kind": "port", "sample": "full workload, CPU oracle"},
                     "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0}, "c_nnz": C.nnz, "products": P})
    print(json.dumps(line), flush=True)
    return 0


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
    from appt_spgemm import matrices as M

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)

    # ---- workload: stencil 64 x 64 x (64 N), B replicated by broadcast from rank 0
    g = 64
    gz = 64 * world
    if rank == 0:
        A = M.stencil27(g, gz=gz)
        sizes = torch.tensor([A.rows, A.nnz], dtype=torch.int64, device=dev)
    else:
        A = None
        sizes = torch.zeros(2, dtype=torch.int64, device=dev)
    t_rep = 0.0
    if world > 1:
        dist.broadcast(sizes, 0)
    rows, nnz = int(sizes[0]), int(sizes[1])
    if rank == 0:
        d_rp = torch.from_numpy(A.row_ptr).to(dev)
        d_ci = torch.from_numpy(A.col_idx).to(dev)
        d_va = torch.from_numpy(A.val).to(dev)
    else:
        d_rp = torch.empty(rows + 1, dtype=torch.int32, device=dev)
        d_ci = torch.empty(nnz, dtype=torch.int32, device=dev)
        d_va = torch.empty(nnz, dtype=torch.float64, device=dev)
    if world > 1:
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for t in (d_rp, d_ci, d_va):
            dist.broadcast(t, 0)
        e1.record()
        torch.cuda.synchronize()
        t_rep = e0.elapsed_time(e1)
        if rank != 0:
            A = M.Csr(rows, rows, d_rp.cpu().numpy(), d_ci.cpu().numpy(), d_va.cpu().numpy())
    torch.cuda.synchronize()

    # ---- row partition balanced by intermediate products (computed by the engine)
    flops = ap.row_products(A, device=local)
    cum = np.concatenate([[0], np.cumsum(flops)])
    total_products = int(cum[-1])
    bounds = [int(np.searchsorted(cum, total_products * r / world, side="left")) for r in range(world)]
    bounds.append(rows)
    bounds[0] = 0
    r0, r1 = bounds[rank], bounds[rank + 1]
    my_products = int(cum[r1] - cum[r0])
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    base_rp = d_rp.data_ptr() + 4 * r0
    blk_nnz = int(A.row_ptr[r1] - A.row_ptr[r0])
    Bspec = (rows, rows, nnz, d_rp.data_ptr(), d_ci.data_ptr(), d_va.data_ptr())

    def step(timing=True):
        res = ap.spgemm_device(r1 - r0, rows, blk_nnz, base_rp, d_ci.data_ptr(), d_va.data_ptr(),
                               B=Bspec, op="ab", method=args.method, stream=sptr, device=local,
                               timing=timing)
        if world > 1:
            mine = torch.tensor([res.nnz], dtype=torch.int64, device=dev)
            allv = torch.empty(world, dtype=torch.int64, device=dev)
            dist.all_gather_into_tensor(allv, mine)
            res.global_offset = int(allv[:rank].sum())
        return res

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        step().free()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    clk = ClockSampler(local)
    clk.start()
    launches0 = ap.kernel_launches()
    step_ms, num_ms, c_nnz = [], [], 0
    stats = None
    for _ in range(args.steps):
        flush.fill_(1)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        res = step()
        ev1.record(stream)
        ev1.synchronize()
        step_ms.append(ev0.elapsed_time(ev1))
        num_ms.append(res.stats["ms_phase"]["numeric"])
        c_nnz = res.nnz
        stats = res.stats
        res.free()
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
        t_total_max, t_num_max = float(tt[0]), float(tt[1])
        pr = torch.tensor([my_products, c_nnz], dtype=torch.int64, device=dev)
        dist.all_reduce(pr)
        all_products, all_cnnz = int(pr[0]), int(pr[1])
    else:
        t_total_max, t_num_max = t_total, t_num
        all_products, all_cnnz = my_products, c_nnz
    value = 2.0 * all_products * args.steps / (t_total_max * 1e-3) / 1e9

    # ---- roofline of the dominant kernel (numeric phase) on this rank's block
    peaks = measured_peaks()
    cbytes = compulsory_bytes(A, r0, r1, c_nnz)
    achieved = cbytes / (t_num * 1e-3) / 1e9
    tr, tr_src = traffic_from_profiles("num_warp_hash_stencil27")

    # ---- e2e through the reference-facing entry point with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = e2e_measure(args, A, r0, r1, rows, world, rank, local, dist, torch)

    # ---- CPU baseline (oracle port) on rank 0 at N = 1
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(A)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_total_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded numpy PCG64 27-point stencil, values U(0.5,1.5))",
            "config": {"workload": WORKLOAD if world == 1 else f"stencil27_64x64x{gz}_AxA",
                       "rows": rows, "nnz_a": nnz, "nnz_c": all_cnnz, "products": all_products,
                       "method": args.method, "parallelism": f"row-sharded x{world}",
                       "l2": "flushed between steps (256 MB write)",
                       "b_replication_ms": t_rep},
            "effective_gbs": cbytes / (t_total_max / args.steps * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": tr,
                         "kernel": "numeric phase (num_warp_hash tiers)",
                         "algorithmic_bytes": cbytes, "avg_ms": t_num,
                         "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"
                         if peaks["source"] == "measured" else "fallback 6.65 TB/s",
                         "traffic_source": tr_src},
            "phase_ms": stats["ms_phase"] if stats else None,
            "bin_rows": stats["bin_rows"] if stats else None,
            "clocks": clocks, "gpu_launches": launches,
            "e2e": e2e, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def e2e_measure(args, A, r0, r1, rows, world, rank, local, dist, torch):
    import appt_spgemm as ap
    if world == 1:
        ap.set_mempool(True, cap_bytes=0)
        nbytes = ap.reference_buffer_bytes(A)
        pinned = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        buf = ap.pack_reference_buffer(A, out=pinned.numpy())
        times = []
        cn = 0
        for it in range(args.warmup + args.steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            C, cr, cc, cn = ap.reference_entry("spgemm_self_product_adaptive", A, buffer=buf,
                                               parse=False)
            t1 = time.perf_counter()
            if cn < 0:
                raise RuntimeError(f"reference entry failed: {ap.last_error()}")
            if it >= args.warmup:
                times.append(t1 - t0)
        t = float(np.mean(times))
        P = int(np.sum(ap.row_products(A, device=local)))
        d2h = ((4 * (A.rows + 1) + 7) & ~7) + ((4 * cn + 7) & ~7) + 8 * cn
        return {"value": 2.0 * P / t / 1e9, "unit": UNIT, "h2d_bytes_per_step": int(nbytes),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": t * 1e3,
                "api": "spgemm_self_product_adaptive (reference signature, pinned host buffers)"}
    # N > 1: native host-buffer call on this rank's row block
    blk = A.__class__(r1 - r0, rows, A.row_ptr[r0:r1 + 1], A.col_idx, A.val)
    times = []
    cnnz = 0
    for it in range(args.warmup + args.steps):
        dist.barrier()
        t0 = time.perf_counter()
        C = ap.spgemm(blk, A, op="ab", device=local)
        t1 = time.perf_counter()
        cnnz = C.nnz
        if it >= args.warmup:
            times.append(t1 - t0)
    t = torch.tensor([float(np.mean(times))], dtype=torch.float64, device=torch.device("cuda", local))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    prods = torch.tensor([int(np.sum(ap.row_products(blk, A, device=local)))], dtype=torch.int64,
                         device=torch.device("cuda", local))
    dist.all_reduce(prods)
    h2d = 4 * (blk.rows + 1) + 12 * blk.nnz + 4 * (A.rows + 1) + 12 * A.nnz
    return {"value": 2.0 * int(prods[0]) / float(t[0]) / 1e9, "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(8 * (blk.rows + 1) + 12 * cnnz),
            "ms_per_step": float(t[0]) * 1e3, "api": "appt_spgemm (host buffers, row block)"}


def cpu_baseline(A):
    import oracle
    P = int(oracle.row_products(A).sum())
    t0 = time.perf_counter()
    oracle.spgemm(A)
    dt = time.perf_counter() - t0
    return {"value": 2.0 * P / dt / 1e9, "unit": UNIT, "cores": oracle.num_threads(),
            "kind": "port", "sample": f"full workload ({A.rows} rows, {P} products), "
                                      f"{dt:.2f} s on the host cores"}


if __name__ == "__main__":
    sys.exit(main())
