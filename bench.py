"""Benchmark of the CQ decode GEMV on B200 (one JSON line on rank 0).

Workload (the HBM-roofline GEMV of the benchmark plan): y = W x with W a CQ4
matrix of 14336 x 4096 (group 128) packed from N(0, 0.02) seed-0 weights and x
one 4096-wide N(0, 1) activation row (seed 1), SDOT int8 mode (per-group int8
activations, int8 centroids, exact int32 per group).  One step = prepare
(rotate + quantise x) + multiply on one of R distinct device copies of W,
cycled so that the working set (R x 30.3 MB) is several times the 126 MB L2;
every launch therefore streams its weights from HBM.

value    = algorithmic bytes of all steps on all ranks / max-over-ranks device time
roofline = the GEMV kernel alone: algorithmic bytes per launch / its mean CUDA-event
           duration, against the measured HBM copy bandwidth
e2e      = the same metric through the reference-facing host call
           (needle2_sdot_linear: host x -> device -> host y, synchronised)
cpu_baseline / --impl reference = the reference's own CPU SDOT path
           (oracle/_ref, compiled from its sources) on this host's cores.

Multi-GPU: each rank runs the same workload on its own GPU (replicas; the
standalone GEMV does not shard), scaling "weak".
"""
from __future__ import annotations

import argparse
import ctypes as ct
import json
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_OUT, K_IN, BITS, GROUP, M_ROWS = 14336, 4096, 4, 128, 1
L2_BYTES = 126 * 1024 * 1024


def algorithmic_bytes(n=N_OUT, k=K_IN, bits=BITS, group=GROUP, m=M_ROWS) -> int:
    """Packed weights + FP16 norms + FP32 input and output: N*(pad*b/8 + 2*pad/G) + 4*M*K + 4*M*N."""
    pad = -(-k // group) * group
    return n * (pad * bits // 8 + 2 * pad // group) + 4 * m * k + 4 * m * n


def peaks():
    try:
        with open(ROOT / "MEASURED_PEAKS.json") as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = max(smax, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def weights():
    from openneedle_b200.quantize import synthetic_matrix
    return synthetic_matrix(N_OUT, K_IN, BITS, GROUP, seed=0)


def activations():
    return np.random.default_rng(1).normal(size=(M_ROWS, K_IN)).astype(np.float32)


# ----------------------------------------------------------- reference arm

def reference_gemv(packed, norms, cb, x, seconds=None, steps=None, warmup=2, copies=4):
    """Times the reference's SdotCQ (prepare + multiply, OpenMP rows) on all host threads.
    Returns (GB/s, seconds per step, steps run, threads, kind)."""
    from oracle import oracle as O
    threads = cpu_threads()
    os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
    y = np.empty((M_ROWS, N_OUT), np.float32)
    if O.ref_available():
        L = O.ref_lib()
        mats = [np.array(packed, copy=True) for _ in range(copies)]
        handles = [L.ref_sdot_new(m.ctypes.data, norms.ctypes.data, N_OUT, K_IN, BITS, GROUP, cb.ctypes.data)
                   for m in mats]
        run = lambda i: L.ref_sdot_run(handles[i % copies], x.ctypes.data, y.ctypes.data, M_ROWS, threads)  # noqa: E731
        kind, used = "reference", threads
    else:
        run = lambda i: O.sdot_linear(packed, norms, (N_OUT, K_IN), BITS, GROUP, cb, x)  # noqa: E731
        kind, used, handles = "port", 1, []
    for i in range(warmup):
        run(i)
    t0 = time.perf_counter()
    n = 0
    while True:
        run(n)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (seconds is not None and el >= seconds):
            break
    el = time.perf_counter() - t0
    if handles:
        for h in handles:
            O.ref_lib().ref_sdot_free(h)
    return algorithmic_bytes() * n / el / 1e9, el / n, n, used, kind


# ------------------------------------------------------------- native arm

class SdotHandle:
    def __init__(self, lib, packed, norms, cb):
        self.lib = lib
        self.h = lib.needle2_sdot_create(packed.ctypes.data, norms.ctypes.data, N_OUT, K_IN, BITS, GROUP,
                                         cb.ctypes.data)
        if not self.h:
            raise RuntimeError(lib.needle2_b200_error().decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.needle2_sdot_destroy(self.h)


def check(status, lib):
    if status:
        raise RuntimeError(lib.needle2_b200_error().decode())


def run_native(args, rank, world, dist):
    import torch
    from openneedle_b200 import build as b
    from openneedle_b200.native import _library

    if rank == 0:
        b.build()
    if dist is not None:
        dist.barrier()
    lib = _library()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    packed, norms, cb = weights()
    x_host = activations()
    bytes_step = algorithmic_bytes()
    per_copy = N_OUT * (packed.shape[1] + 2 * norms.shape[1])
    copies = args.copies or max(4, -(-4 * L2_BYTES // per_copy))  # working set >= 4x L2
    handles = [SdotHandle(lib, packed, norms, cb) for _ in range(copies)]
    x = torch.from_numpy(x_host).to(dev)
    y = torch.empty(M_ROWS, N_OUT, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step(i):
        h = handles[i % copies].h
        check(lib.needle2_sdot_prepare_device(h, x.data_ptr(), M_ROWS, sp), lib)
        check(lib.needle2_sdot_multiply_device(h, y.data_ptr(), M_ROWS, sp), lib)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        end.record(stream)
        torch.cuda.synchronize(dev)
    elapsed_ms = start.elapsed_time(end)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)

    # kernel alone: events around each multiply launch
    kstart = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    kend = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        h = handles[i % copies].h
        check(lib.needle2_sdot_prepare_device(h, x.data_ptr(), M_ROWS, sp), lib)
        kstart[i].record(stream)
        check(lib.needle2_sdot_multiply_device(h, y.data_ptr(), M_ROWS, sp), lib)
        kend[i].record(stream)
    torch.cuda.synchronize(dev)
    kernel_ms = float(np.mean([a.elapsed_time(b_) for a, b_ in zip(kstart, kend)]))

    # end to end through the reference-facing host call
    e2e_s = float("nan")
    if not args.skip_e2e:
        lib_y = np.empty((M_ROWS, N_OUT), np.float32)
        for i in range(3):
            check(lib.needle2_sdot_linear_checked(handles[i % copies].h, x_host.ctypes.data, lib_y.ctypes.data,
                                                  M_ROWS), lib)
        e2e_steps = max(args.steps, 20)
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            check(lib.needle2_sdot_linear_checked(handles[i % copies].h, x_host.ctypes.data, lib_y.ctypes.data,
                                                  M_ROWS), lib)
        e2e_s = (time.perf_counter() - t0) / e2e_steps

    # FP32 mode beside it (same weights, same copies)
    fp32 = None if args.skip_fp32 else run_fp32_mode(lib, packed, norms, cb, x, y, copies, stream, args, dev)

    t = torch.tensor([elapsed_ms, kernel_ms, e2e_s], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, kernel_ms, e2e_s = t.tolist()
    total_bytes = bytes_step * args.steps * world
    hbm, peak_kind = peaks()
    achieved = bytes_step / (kernel_ms * 1e-3) / 1e9
    result = {
        "metric": "cq4_gemv_hbm_gbs",
        "value": total_bytes / (elapsed_ms * 1e-3) / 1e9,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "i8",
        "data": "synthetic",
        "config": {"workload": f"cq4_sdot_gemv_m{M_ROWS}_{N_OUT}x{K_IN}", "bits": BITS, "group": GROUP,
                   "M": M_ROWS, "N": N_OUT, "K": K_IN, "mode": "sdot-int8", "weight_copies": copies,
                   "working_set_bytes": per_copy * copies,
                   "l2": "inputs larger than L2: distinct weight copies cycled, working set >= 4x L2",
                   "parallelism": f"replicas{world}", "bytes_per_step": bytes_step},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": peak_kind, "kernel": "cq_gemv_kernel<I8,4>", "kernel_ms": kernel_ms,
                     "traffic": profiled_traffic("cq_gemv_i8")},
        "e2e": None if args.skip_e2e else {
            "value": bytes_step / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 4 * M_ROWS * K_IN,
            "d2h_bytes_per_step": 4 * M_ROWS * N_OUT, "ms_per_step": e2e_s * 1e3},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
        "fp32_mode": fp32,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, sec, n, threads, kind = reference_gemv(packed, norms, cb, x_host, seconds=args.cpu_seconds)
        result["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                                  "sample": f"{n} SDOT GEMVs of the same 14336x4096 CQ4 matrix (4 host copies "
                                            f"cycled), {sec * 1e3:.2f} ms each, ~{args.cpu_seconds:.0f} s bound; "
                                            "x86 runs the reference's portable (non-NEON) branches"}
    return result


def run_fp32_mode(lib, packed, norms, cb, x, y, copies, stream, args, dev):
    import torch
    sp = stream.cuda_stream
    hs = []
    for _ in range(copies):
        h = lib.needle2_cq_create(packed.ctypes.data, norms.ctypes.data, N_OUT, K_IN, BITS, GROUP, cb.ctypes.data)
        if not h:
            raise RuntimeError(lib.needle2_b200_error().decode())
        hs.append(h)
    try:
        for i in range(args.warmup):
            check(lib.needle2_cq_prepare_device(hs[i % copies], x.data_ptr(), M_ROWS, sp), lib)
            check(lib.needle2_cq_multiply_device(hs[i % copies], y.data_ptr(), M_ROWS, sp), lib)
        ks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ke = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            h = hs[i % copies]
            check(lib.needle2_cq_prepare_device(h, x.data_ptr(), M_ROWS, sp), lib)
            ks[i].record(stream)
            check(lib.needle2_cq_multiply_device(h, y.data_ptr(), M_ROWS, sp), lib)
            ke[i].record(stream)
        torch.cuda.synchronize(dev)
        kms = float(np.mean([a.elapsed_time(b) for a, b in zip(ks, ke)]))
    finally:
        for h in hs:
            lib.needle2_cq_destroy(h)
    hbm, _ = peaks()
    gbs = algorithmic_bytes() / (kms * 1e-3) / 1e9
    return {"kernel": "cq_gemv_kernel<FP32,4>", "kernel_ms": kms, "achieved_gbs": gbs, "frac": gbs / hbm}


def profiled_traffic(tag):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    for f in sorted((ROOT / "profiles").glob(f"{tag}*.md")):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
        if m:
            return float(m.group(1))
    return None


def run_reference_arm(args, rank, world):
    if rank != 0:
        return None
    packed, norms, cb = weights()
    x = activations()
    gbs, sec, n, threads, kind = reference_gemv(packed, norms, cb, x, steps=args.steps, warmup=args.warmup)
    return {
        "impl": "reference", "metric": "cq4_gemv_hbm_gbs", "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8", "data": "synthetic",
        "config": {"workload": f"cq4_sdot_gemv_m{M_ROWS}_{N_OUT}x{K_IN}", "bits": BITS, "group": GROUP, "M": M_ROWS,
                   "N": N_OUT, "K": K_IN, "mode": "sdot-int8", "parallelism": "host cores (OpenMP rows)"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{n} steps of the reference SdotCQ GEMV over 4 host copies of the matrix"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--copies", type=int, default=0, help="weight copies (default: working set >= 4x L2)")
    ap.add_argument("--skip-fp32", action="store_true", help="omit the FP32-mode side measurement")
    ap.add_argument("--skip-e2e", action="store_true", help="omit the host-buffer end-to-end measurement")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if args.impl == "reference":
        result = run_reference_arm(args, rank, world)
    else:
        if world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        try:
            result = run_native(args, rank, world, dist)
        finally:
            if dist is not None:
                dist.destroy_process_group()
    if rank == 0 and result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
