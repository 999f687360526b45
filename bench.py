"""Benchmark of OpenNeedle's quantized hot path on B200 (one JSON line on rank 0).

Headline (the batched-decode half of the metric): the
Needle-2 decoder (d 512, 12 layers, 8 query / 4 KV heads x 64, vocab 32768,
engram sites at layers 2 and 9) as the reference's NeedleModel default init
(seed 0) packed by the reference's quantizer in the release scheme (CQ4
embedding and mHC, CQ2 projections and engram tables), FP32 matmul mode,
INT8 KV.  1024 sessions with 256-token prompts (default_rng(0) tokens) are
prefilled (untimed), then every step decodes one greedy token for every
session.  Sessions are split evenly over the GPUs (one process per GPU,
weights replicated, no collective), so the total work is fixed: "strong".

value     sessions * K steps / max-over-ranks device time of K steps (one
          needle2_batch_decode_greedy_device call between CUDA events)
roofline  the decode step's dominant stage (KV store + attention over the
          INT8 cache, 12 layers), from the engine's per-stage CUDA-event timers
          in a profiled pass: its algorithmic bytes / its time, against the
          measured HBM copy bandwidth (MEASURED_PEAKS.json)
e2e       the same metric through needle2_batch_step from host buffers: each
          step's tokens copied in and its greedy tokens read back
cpu_baseline / --impl reference
          the reference's own engine (needle2/native.py NativeEngine on its CPU
          library built from its sources, oracle/_ref, all host threads, INT8
          KV): decode steps of one session after a 256-token prefill; it serves
          one sequence per engine, so its tokens/s is per sequence served.

Side lines: cq_gemv (the HBM-roofline decode GEMV of 17 fused 14336x4096 CQ4
matrices, SDOT mode, with its own roofline and CPU baseline), the config-3
prefill GEMMs, config-4 INT8 KV attention, and on 2+ GPUs the N-sharded
14336x4096 GEMM with its all-gather.
"""
from __future__ import annotations

import argparse
import ctypes as ct
import json
import os
import re
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_OUT, K_IN, BITS, GROUP, M_ROWS, COPIES = 14336, 4096, 4, 128, 1, 17
L2_BYTES = 126 * 1024 * 1024


def matrix_bytes(n=N_OUT, k=K_IN, bits=BITS, group=GROUP) -> int:
    """Packed weights + FP16 norms of one matrix: N*(pad*b/8 + 2*pad/G)."""
    pad = -(-k // group) * group
    return n * (pad * bits // 8 + 2 * pad // group)


def step_bytes(copies=COPIES, m=M_ROWS) -> int:
    """Algorithmic bytes of one fused step: R matrices, the FP32 input once, R FP32 outputs."""
    return copies * (matrix_bytes() + 4 * m * N_OUT) + 4 * m * K_IN


def peaks():
    try:
        with open(ROOT / "MEASURED_PEAKS.json") as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle-reason samples taken through NVML every ~1 ms
    during the timed region (the fields of nvidia-smi's clocks query)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self._max = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001 - clocks are then reported as unavailable
            self._nvml = None
        return self

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                sm = n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((float(sm), float(self._max), int(reasons)))
            except Exception:  # noqa: BLE001
                break
            time.sleep(0.001)

    def __exit__(self, *exc):
        self._stop.set()
        if getattr(self, "thread", None):
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": "nvml"}
        mask = 0
        for s in self.samples:
            mask |= s[2]
        return {"sm_mhz": float(np.median([s[0] for s in self.samples])), "sm_max_mhz": self.samples[0][1],
                "reasons": sorted(k for k, bit in self.REASONS.items() if mask & bit),
                "samples": len(self.samples), "source": "nvml, ~1 ms period"}


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def ref_quantize():
    """The reference's own CQ packer (needle2/quantize.py, as BASELINE config 1
    prescribes), from the reference package: NEEDLE2_REFERENCE_SRC, default the
    copy pip installed into baseline/_ref.  It only builds the synthetic inputs."""
    root = Path(os.environ.get("NEEDLE2_REFERENCE_SRC", str(ROOT / "baseline" / "_ref")))
    if not (root / "needle2" / "quantize.py").is_file():
        raise SystemExit(f"reference package not found under {root} (needed to pack the synthetic weights); "
                         "install it into baseline/_ref or set NEEDLE2_REFERENCE_SRC")
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    from needle2 import quantize
    return quantize


def synthetic_matrix(rows, cols, bits, group, seed):
    """W ~ N(0, 0.02) from default_rng(seed), packed by the reference's quantizer."""
    q = ref_quantize()
    w = np.random.default_rng(seed).normal(0.0, 0.02, (rows, cols)).astype(np.float32)
    packed, norms = q.quantize_matrix(w, bits, group)
    return packed, norms, q.codebook(bits, group)


def weights():
    return synthetic_matrix(N_OUT, K_IN, BITS, GROUP, seed=0)


def activations():
    return np.random.default_rng(1).normal(size=(M_ROWS, K_IN)).astype(np.float32)


def profiled_traffic(tag):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    for f in sorted((ROOT / "profiles").glob(f"{tag}*.md")):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
        if m:
            return float(m.group(1))
    return None


def workload_config(copies, world):
    return {"workload": f"cq4_sdot_gemv_fused{copies}x{N_OUT}x{K_IN}_m{M_ROWS}", "bits": BITS, "group": GROUP,
            "M": M_ROWS, "N": N_OUT, "K": K_IN, "matrices_per_step": copies, "mode": "sdot-int8",
            "weight_bytes_per_step": copies * matrix_bytes(),
            "l2": f"inputs larger than L2: each step streams {copies} distinct 30 MB matrices",
            "parallelism": f"replicas{world}", "bytes_per_step": step_bytes(copies)}


# ----------------------------------------------------------- reference arm

def reference_gemv(packed, norms, cb, x, seconds=None, steps=None, warmup=2, host_copies=4):
    """Times the reference's SdotCQ (prepare + multiply, OpenMP rows) on all host
    threads.  One sample = one GEMV of one 14336x4096 matrix (host copies cycled);
    the rate in GB/s counts the same algorithmic bytes per matrix as the GPU arm.
    Returns (GB/s, seconds per GEMV, GEMVs run, threads, kind)."""
    from oracle import oracle as O
    threads = cpu_threads()
    os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
    y = np.empty((M_ROWS, N_OUT), np.float32)
    if O.ref_available():
        L = O.ref_lib()
        mats = [np.array(packed, copy=True) for _ in range(host_copies)]
        handles = [L.ref_sdot_new(m.ctypes.data, norms.ctypes.data, N_OUT, K_IN, BITS, GROUP, cb.ctypes.data)
                   for m in mats]

        def run(i):
            L.ref_sdot_run(handles[i % host_copies], x.ctypes.data, y.ctypes.data, M_ROWS, threads)
        kind, used = "reference", threads
    else:
        handles = []

        def run(i):
            O.sdot_linear(packed, norms, (N_OUT, K_IN), BITS, GROUP, cb, x)
        kind, used = "port", 1
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
    for h in handles:
        O.ref_lib().ref_sdot_free(h)
    per_matrix = matrix_bytes() + 4 * M_ROWS * (N_OUT + K_IN)
    return per_matrix * n / el / 1e9, el / n, n, used, kind


def gemv_reference_arm(args, rank, world):
    if rank != 0:
        return None
    packed, norms, cb = weights()
    x = activations()
    gbs, sec, n, threads, kind = reference_gemv(packed, norms, cb, x, steps=args.steps, warmup=args.warmup)
    return {
        "impl": "reference", "metric": "cq4_gemv_hbm_gbs", "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "i8", "data": "synthetic", "config": workload_config(COPIES, world),
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"each step one reference SdotCQ GEMV of one 14336x4096 CQ4 matrix (4 host "
                                   f"copies cycled), {n} steps; a bounded sample of the {COPIES}-matrix step"},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------- native arm

def check(status, lib):
    if status:
        raise RuntimeError(lib.needle2_b200_error().decode())


def create(lib, packed, norms, cb, sdot):
    fn = lib.needle2_sdot_create if sdot else lib.needle2_cq_create
    h = fn(packed.ctypes.data, norms.ctypes.data, N_OUT, K_IN, BITS, GROUP, cb.ctypes.data)
    if not h:
        raise RuntimeError(lib.needle2_b200_error().decode())
    return h


def kernel_ms(lib, handles, x, yp, stream, sdot, n):
    """Mean CUDA-event duration of the fused GEMV launch alone (prepare outside)."""
    import torch
    sp = stream.cuda_stream
    hp = (ct.c_void_p * len(handles))(*handles)
    prep = lib.needle2_sdot_prepare_device if sdot else lib.needle2_cq_prepare_device
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    for i in range(n):
        check(prep(handles[0], x.data_ptr(), M_ROWS, sp), lib)
        starts[i].record(stream)
        check(lib.needle2_cq_multiply_many_device(hp, len(handles), yp, M_ROWS, int(sdot), sp), lib)
        ends[i].record(stream)
    torch.cuda.synchronize()
    return float(np.mean([a.elapsed_time(b) for a, b in zip(starts, ends)]))


def _gemm_ms(lib, dev, stream, packed, norms, cb, m, n, k, bits, reps):
    """Mean kernel time (ms) of one M x K x N product in the int8 (SDOT) mode and
    in the FP32 mode: the quantised / split activations are prepared outside the
    timed launches, the weights are decoded once before them."""
    import torch
    x = torch.randn(m, k, device=dev)
    y = torch.empty(m, n, device=dev)
    sp = stream.cuda_stream
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = []
    for create, linear, prep, mult, destroy in (
            (lib.needle2_sdot_create, lib.needle2_sdot_linear_device, lib.needle2_sdot_prepare_device,
             lib.needle2_sdot_multiply_device, lib.needle2_sdot_destroy),
            (lib.needle2_cq_create, lib.needle2_cq_linear_device, lib.needle2_cq_prepare_device,
             lib.needle2_cq_multiply_device, lib.needle2_cq_destroy)):
        h = create(packed.ctypes.data, norms.ctypes.data, n, k, bits, GROUP, cb.ctypes.data)
        if not h:
            raise RuntimeError(lib.needle2_b200_error().decode())
        check(linear(h, x.data_ptr(), y.data_ptr(), m, sp), lib)   # decodes the weights once
        check(prep(h, x.data_ptr(), m, sp), lib)
        for _ in range(3):
            check(mult(h, y.data_ptr(), m, sp), lib)
        a.record(stream)
        for _ in range(reps):
            check(mult(h, y.data_ptr(), m, sp), lib)
        b.record(stream)
        torch.cuda.synchronize(dev)
        out.append(a.elapsed_time(b) / reps)
        destroy(h)
    return out


def _bf16_peak():
    try:
        with open(ROOT / "MEASURED_PEAKS.json") as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return None


def prefill_gemm(lib, dev, stream, reps=20):
    """Config 3's largest case on the int8 prefill GEMM: x[2048][4096] against a
    CQ4 8192 x 4096 matrix (group 128); the GEMM kernel alone (quantised input
    prepared outside the timed launches), against twice the measured bf16 dense
    rate (B200 issues int8 MMAs at twice the bf16 rate)."""
    m, n, k = 2048, 8192, 4096
    packed, norms, cb = synthetic_matrix(n, k, 4, GROUP, seed=3)
    ms, fms = _gemm_ms(lib, dev, stream, packed, norms, cb, m, n, k, 4, reps)
    tops = 2.0 * m * n * k / (ms * 1e-3) / 1e12
    bf16 = _bf16_peak()
    peak = 2 * bf16 if bf16 else 2 * 1590.0
    ftf = 2.0 * m * n * k / (fms * 1e-3) / 1e12
    fp32 = {"kernel": "cq_gemm_f32x3_kernel (tcgen05 kind::f16, bf16 hi/lo split, 3 MMAs per K step, 128x256 tiles)",
            "kernel_ms": fms, "achieved": ftf, "unit": "TFLOP/s", "peak": bf16 or 1590.0,
            "frac": ftf / (bf16 or 1590.0), "tensor_pipe_frac": 3 * ftf / (bf16 or 1590.0),
            "note": "FP32-equivalent flops against the measured bf16 dense rate; three bf16 products per FP32 "
                    "product, so 1/3 is this kernel's ceiling (tensor_pipe_frac counts all three)",
            "call": "needle2_cq_multiply_device (split activations + GEMM)"}
    return {"config": "M=2048 x K=4096 x N=8192, CQ4 group 128, int8 (SDOT) mode, bit-exact epilogue",
            "kernel": "cq_gemm_i8_kernel (tcgen05 kind::i8, 128x192 tiles, TMA 128B-swizzled)",
            "kernel_ms": ms, "achieved": tops, "unit": "TOP/s", "bound": "tensor", "peak": peak,
            "frac": tops / peak, "peak_source": "2 x measured bf16 dense" if bf16 else "2 x fallback bf16 dense",
            "fp32_mode": fp32}


def prefill_gemm_sweep(lib, dev, stream, reps=10):
    """Config 3's grid: M = 2048 against N in {2048, 8192, 11008} x K in
    {512, 2048, 4096}, CQ4 and CQ2, both modes; kernel ms per shape.  The packed
    codes and group norms are seeded random bytes / half values of the real
    layout: the kernels' time does not depend on the values (parity is covered by
    the tests), and quantising 18 matrices on the host would take minutes."""
    codebook = ref_quantize().codebook
    rng = np.random.default_rng(5)
    m = 2048
    bf16 = _bf16_peak() or 1590.0
    rows = []
    for bits in (4, 2):
        cb = np.ascontiguousarray(codebook(bits, GROUP), dtype=np.float32)
        for n in (2048, 8192, 11008):
            for k in (512, 2048, 4096):
                packed = rng.integers(0, 256, (n, k * bits // 8), dtype=np.uint8)
                norms = rng.uniform(0.15, 0.3, (n, k // GROUP)).astype(np.float16)
                ms, fms = _gemm_ms(lib, dev, stream, packed, norms, cb, m, n, k, bits, reps)
                ops = 2.0 * m * n * k
                rows.append({"bits": bits, "n": n, "k": k, "int8_ms": round(ms, 4),
                             "int8_frac": round(ops / (ms * 1e-3) / 1e12 / (2 * bf16), 3),
                             "fp32_ms": round(fms, 4),
                             "fp32_frac": round(ops / (fms * 1e-3) / 1e12 / bf16, 3)})
    return {"m": m, "group": GROUP, "reps": reps,
            "frac_note": "int8 against 2 x measured bf16 dense, fp32 (FP32-equivalent flops) against measured "
                         "bf16 dense", "shapes": rows}


def attention_decode(dev, stream, lengths=(512, 2048, 4096), reps=20):
    """Config 4: INT8 KV decode attention for 256 sessions sharing a 384-token
    prefix (H=8, KV=4, HD=64), one decode step (store the new token, attend)
    per session at each context length L.  Bytes = unique KV read (prefix once,
    each session's own L - 384 slots) x (2*KV*HD + 8*KV) + q, out, new k, v."""
    import torch
    from openneedle_b200.attention import KVCache
    sessions, heads, kvh, hd, prefix, max_seq = 256, 8, 4, 64, 384, max(lengths)
    kv = KVCache(sessions, heads, kvh, hd, max_seq, window=0, prefix_len=prefix)
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    kw = kvh * hd
    kv.set_prefix_device(torch.randn(prefix, kw, device=dev, generator=g),
                         torch.randn(prefix, kw, device=dev, generator=g), stream)
    ids = np.arange(sessions, dtype=np.int32)
    k_tok = torch.randn(sessions, kw, device=dev, generator=g)
    v_tok = torch.randn(sessions, kw, device=dev, generator=g)
    q = torch.randn(sessions, heads * hd, device=dev, generator=g)
    out = torch.empty_like(q)
    slot_bytes = 2 * kvh * hd + 8 * kvh
    # prefill: every session's 128 tokens on top of the shared prefix (store, then
    # causal attention per token), repeated over the same positions
    t = 128
    qp = torch.randn(sessions, t, heads * hd, device=dev, generator=g)
    kp = torch.randn(sessions, t, kw, device=dev, generator=g)
    vp = torch.randn(sessions, t, kw, device=dev, generator=g)
    op = torch.empty_like(qp)
    starts = np.full(sessions, prefix, np.int32)
    for _ in range(2):
        kv.prefill_device(ids, starts, t, qp, kp, vp, op, stream)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(5):
        kv.prefill_device(ids, starts, t, qp, kp, vp, op, stream)
    b.record(stream)
    torch.cuda.synchronize(dev)
    pms = a.elapsed_time(b) / 5
    prefill = {"tokens_per_session": t, "ms": pms, "tokens_per_s": sessions * t / (pms * 1e-3),
               "note": "256 sessions x 128 new tokens after the 384-token prefix; causal, store-then-attend"}
    rows, filled = [], prefix
    for length in lengths:
        # fill every session's cache up to position length - 2 (fresh values per position)
        while filled < length - 1:
            k_tok.normal_(generator=g)
            v_tok.normal_(generator=g)
            kv.store_device(ids, np.full(sessions, filled, np.int32), k_tok, v_tok, stream)
            filled += 1
        pos = np.full(sessions, length - 1, np.int32)
        for _ in range(3):
            kv.decode_device(ids, pos, q, k_tok, v_tok, out, stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            kv.decode_device(ids, pos, q, k_tok, v_tok, out, stream)
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b) / reps
        unique = (prefix + sessions * (length - prefix)) * slot_bytes + sessions * 4 * (2 * heads * hd + 2 * kw)
        gbs = unique / (ms * 1e-3) / 1e9
        rows.append({"context": length, "ms_per_step": ms, "tokens_per_s": sessions / (ms * 1e-3),
                     "algorithmic_bytes": unique, "achieved_gbs": gbs, "frac": gbs / peaks()[0]})
    del kv
    return {"config": "256 sessions, H=8, KV=4, HD=64, shared 384-token prefix, one decode step per session",
            "kernels": "kv_quantize_kernel + attn_stream_kernel + attn_combine_kernel (split-K flash decode)",
            "bound": "hbm", "peak": peaks()[0], "unit": "GB/s", "by_context": rows, "prefill": prefill}


def sharded_gemm(dev, stream, world, dist, packed, norms, cb, m=2048, reps=10):
    """Config 5b: the 14336 x 4096 CQ4 matrix N-sharded over the ranks (int8
    mode, M = 2048 activation rows), its outputs all-gathered into every rank's
    [M][N].  Times (max over ranks, CUDA events): the all-gather fused into the
    GEMM epilogue (peer stores over NVLink, then a tiny all-reduce as the
    barrier), a local GEMM followed by NCCL's all_gather_into_tensor, and the
    local GEMM alone.  Each rank sends M * N/world * 4 bytes to every other rank."""
    import torch
    from openneedle_b200.sharded import ShardedSdot
    sh = ShardedSdot(packed, norms, (N_OUT, K_IN), BITS, GROUP, cb, max_batch=m, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    x = torch.randn(m, K_IN, device=dev, generator=g)

    def timed(fn):
        for _ in range(3):
            fn(x, stream)
        dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn(x, stream)
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / reps

    fused = timed(sh.forward)
    nccl = timed(sh.forward_nccl)
    local = timed(sh.forward_local)
    t = torch.tensor([fused, nccl, local], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    fused, nccl, local = t.tolist()
    # correctness on every rank: the fused and the NCCL all-gather against the
    # whole matrix on one GPU (same int8 GEMM per row, so bit for bit)
    from openneedle_b200.native import DeviceMatrix
    whole = DeviceMatrix(packed, norms, (N_OUT, K_IN), BITS, GROUP, cb)
    with torch.cuda.stream(stream):
        y_single = torch.empty(m, N_OUT, device=dev)
        whole.sdot.linear_device(x, y_single, stream)
        y_fused = sh.forward(x, stream).clone()
        y_nccl = sh.forward_nccl(x, stream).clone()
    torch.cuda.synchronize(dev)
    flags = torch.tensor([float(torch.equal(y_fused, y_single)), float(torch.equal(y_nccl, y_single))],
                         device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    match_fused, match_nccl = (bool(v) for v in flags.tolist())
    whole.close()
    del y_single, y_fused, y_nccl
    sent = m * sh.ns * 4 * (world - 1)
    flops = 2.0 * m * N_OUT * K_IN
    res = {"config": f"{N_OUT}x{K_IN} CQ4 int8 mode, M={m}, {sh.ns} rows per GPU, outputs all-gathered to every GPU",
           "fused_ms": fused, "nccl_ms": nccl, "local_gemm_ms": local,
           "fused_top_s": flops / (fused * 1e-3) / 1e12, "nccl_top_s": flops / (nccl * 1e-3) / 1e12,
           "nvlink_bytes_sent_per_rank": sent, "fused_send_gbs_per_rank": sent / (fused * 1e-3) / 1e9,
           "match": match_fused and match_nccl, "match_fused": match_fused, "match_nccl": match_nccl,
           "match_against": "the whole matrix's int8 GEMM on one GPU, bitwise, on every rank",
           "timing": "max over ranks; each call = prepare + GEMM (+ exchange); fused includes the barrier all-reduce"}
    sh.close()
    return res


def gemv_native(args, rank, world, dist):
    import torch
    from openneedle_b200.native import _library

    lib = _library()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    packed, norms, cb = weights()
    x_host = activations()
    copies = args.copies or COPIES
    handles = [create(lib, packed, norms, cb, True) for _ in range(copies)]
    hp = (ct.c_void_p * copies)(*handles)
    x = torch.from_numpy(x_host).to(dev)
    ys = torch.empty(copies, M_ROWS, N_OUT, device=dev)
    yp = (ct.c_void_p * copies)(*[ys[i].data_ptr() for i in range(copies)])
    stream = torch.cuda.current_stream(dev)
    bytes_step = step_bytes(copies)

    def step(sp):
        check(lib.needle2_cq_linear_many_device(hp, copies, x.data_ptr(), yp, M_ROWS, 1, sp), lib)

    for _ in range(args.warmup):
        step(stream.cuda_stream)
    torch.cuda.synchronize(dev)
    # K timed steps captured once into a CUDA graph and replayed once; the
    # kernels inside chain by programmatic dependent launch
    graph_stream = torch.cuda.Stream(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(graph_stream):
        with torch.cuda.graph(graph, stream=graph_stream):
            for _ in range(args.steps):
                step(graph_stream.cuda_stream)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        start.record(stream)
        graph.replay()
        end.record(stream)
        torch.cuda.synchronize(dev)
    elapsed_ms = start.elapsed_time(end)
    del graph
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)

    n_kernel = max(5, min(args.steps, 40))
    fused_ms = kernel_ms(lib, handles, x, yp, stream, True, n_kernel)
    single_ms = kernel_ms(lib, handles[:1], x, yp, stream, True, n_kernel)
    e2e = None
    if not args.skip_e2e:
        # the step's input and outputs in page-locked host memory (torch's pinned allocator)
        xp = torch.empty(M_ROWS, K_IN, dtype=torch.float32, pin_memory=True)
        xp.copy_(torch.from_numpy(x_host))
        ys_pinned = [torch.empty(M_ROWS, N_OUT, dtype=torch.float32, pin_memory=True) for _ in range(copies)]
        yhp = (ct.c_void_p * copies)(*[a.data_ptr() for a in ys_pinned])
        for _ in range(3):
            check(lib.needle2_cq_linear_many_checked(hp, copies, xp.data_ptr(), yhp, M_ROWS, 1), lib)
        n_e2e = max(10, min(args.steps, 100))
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            check(lib.needle2_cq_linear_many_checked(hp, copies, xp.data_ptr(), yhp, M_ROWS, 1), lib)
        e2e_s = (time.perf_counter() - t0) / n_e2e
        e2e = {"value": bytes_step / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 4 * M_ROWS * K_IN,
               "d2h_bytes_per_step": 4 * M_ROWS * N_OUT * copies, "ms_per_step": e2e_s * 1e3,
               "call": "needle2_cq_linear_many_checked (page-locked host buffers: x copied in, the GEMV stores "
                       "its outputs straight into the host buffers; synchronised)"}
        # the same call from pageable numpy buffers (the reference's own callers)
        ys_np = [np.empty((M_ROWS, N_OUT), np.float32) for _ in range(copies)]
        ynp = (ct.c_void_p * copies)(*[a.ctypes.data for a in ys_np])
        for _ in range(3):
            check(lib.needle2_cq_linear_many_checked(hp, copies, x_host.ctypes.data, ynp, M_ROWS, 1), lib)
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            check(lib.needle2_cq_linear_many_checked(hp, copies, x_host.ctypes.data, ynp, M_ROWS, 1), lib)
        pg_s = (time.perf_counter() - t0) / n_e2e
        e2e["pageable"] = {"value": bytes_step / pg_s / 1e9, "unit": "GB/s", "ms_per_step": pg_s * 1e3}

    fp32 = None
    if not args.skip_fp32:
        fh = [create(lib, packed, norms, cb, False) for _ in range(copies)]
        fhp = (ct.c_void_p * copies)(*fh)
        for _ in range(3):
            check(lib.needle2_cq_linear_many_device(fhp, copies, x.data_ptr(), yp, M_ROWS, 0, stream.cuda_stream), lib)
        fms = kernel_ms(lib, fh, x, yp, stream, False, n_kernel)
        # the other FP32 GEMV kernels on the same launch, for comparison
        others = {}
        for kind, name, kern in ((1, "slot_kernel", "cq_gemv_kernel<FP32,CQ4,G128,M1> (group per lane)"),
                                 (2, "row_kernel", "cq_gemv_rows_kernel<CQ4,G128,M1> (row per lane, no table)")):
            prev = lib.needle2_b200_set_f32_gemv(kind)
            kernel_ms(lib, fh, x, yp, stream, False, 3)
            oms = kernel_ms(lib, fh, x, yp, stream, False, n_kernel)
            lib.needle2_b200_set_f32_gemv(prev)
            others[name] = {"kernel": kern, "kernel_ms": oms, "achieved_gbs": bytes_step / (oms * 1e-3) / 1e9}
        for h in fh:
            lib.needle2_cq_destroy(h)
        gbs = bytes_step / (fms * 1e-3) / 1e9
        fp32 = {"kernel": f"cq_gemv_ptab_kernel<CQ4,G128> (product table, clusters of 8 CTAs) fused over {copies} "
                          "matrices",
                "kernel_ms": fms, "achieved_gbs": gbs, "frac": gbs / peaks()[0], **others}

    t = torch.tensor([elapsed_ms, fused_ms, single_ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, fused_ms, single_ms = t.tolist()
    hbm, peak_kind = peaks()
    achieved = bytes_step / (fused_ms * 1e-3) / 1e9
    single_gbs = (matrix_bytes() + 4 * M_ROWS * (N_OUT + K_IN)) / (single_ms * 1e-3) / 1e9
    result = {
        "metric": "cq4_gemv_hbm_gbs",
        "value": bytes_step * args.steps * world / (elapsed_ms * 1e-3) / 1e9,
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
        "config": workload_config(copies, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_source": peak_kind,
                     "kernel": f"cq_gemv_frag_kernel<CQ4,G128,M1,sign-split> (mma.sync s8, fragment-order weights) fused over {copies} matrices",
                     "kernel_ms": fused_ms, "traffic": profiled_traffic("cq_gemv_frag_sdot_fused")},
        "single_matrix": {"kernel_ms": single_ms, "achieved_gbs": single_gbs, "frac": single_gbs / hbm,
                          "note": "one 14336x4096 matrix per launch (launch and DRAM ramp overheads included)"},
        "e2e": e2e,
        "gpu_launches": 2 * args.steps,
        "timing": "K steps captured in one CUDA graph, replayed once between CUDA events on the launching stream",
        "clocks": clocks.summary(),
        "fp32_mode": fp32,
    }
    for h in handles:
        lib.needle2_sdot_destroy(h)
    if not args.skip_gemm:
        result["prefill_gemm"] = prefill_gemm(lib, dev, stream)
        if world == 1 and not args.skip_sweep:
            result["prefill_gemm_sweep"] = prefill_gemm_sweep(lib, dev, stream)
    if not args.skip_attention:
        result["attention_decode"] = attention_decode(dev, stream)
    if world > 1 and not args.skip_sharded:
        # a side line: a failure here is reported in it, the headline stands
        try:
            result["sharded_gemm"] = sharded_gemm(dev, stream, world, dist, packed, norms, cb)
        except Exception as e:  # noqa: BLE001
            result["sharded_gemm"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, sec, n, threads, kind = reference_gemv(packed, norms, cb, x_host, seconds=args.cpu_seconds)
        result["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind,
                                  "sample": f"{n} reference SdotCQ GEMVs of one 14336x4096 CQ4 matrix (4 host copies "
                                            f"cycled), {sec * 1e3:.1f} ms each, ~{args.cpu_seconds:.0f} s bound; x86 "
                                            "runs the reference's portable (non-NEON) branches"}
    return result


# ------------------------------------------------------ config-5 decoder

DEC_SESSIONS, DEC_PROMPT, DEC_VOCAB = 1024, 256, 32768
DEC_CONFIG = dict(vocab_size=DEC_VOCAB, d_model=512, num_heads=8, num_kv_heads=4, num_layers=12, head_dim=64,
                  max_seq_len=4096, kv_window=0, engram_layers=(2, 9))


def decoder_archive(seed: int = 0):
    """BASELINE config 5 as an in-memory archive: the reference's
    NeedleModel(config) default init under torch.manual_seed(seed)
    (needle2/model.py:266-287; N(0, 0.02) matrices), packed by the reference's
    quantizer in its release scheme (CQ4 embedding and mHC projections, CQ2
    attention/engram projections and engram tables, FP32 elsewhere) into its
    TensorRecord objects."""
    from types import SimpleNamespace

    import torch
    Q = ref_quantize()
    from needle2 import archive as A
    from needle2 import model as M
    torch.manual_seed(seed)
    model = M.NeedleModel(M.NeedleConfig(**DEC_CONFIG))
    records = {}
    for name, t in model.canonical_state_dict().items():
        a = t.detach().numpy().astype(np.float32)
        if a.ndim == 2 and (name == "embedding" or name.startswith("mhc_phi") or name.endswith(("_proj", ".tables"))):
            bits = 4 if name == "embedding" or name.startswith("mhc_phi") else 2
            p, n = Q.quantize_matrix(a, bits, 128)
            records[name] = A.TensorRecord(name, A.CQ, a.shape, p.tobytes() + n.tobytes(), 128, bits,
                                           Q.codebook(bits, 128))
        else:
            records[name] = A.TensorRecord(name, A.FP32, a.shape, a.tobytes())
    meta = model.config.to_dict()
    meta["hada_n"] = 1 << (meta["d_model"] - 1).bit_length()
    return SimpleNamespace(metadata=meta, tensors=records)


def decoder_prompts():
    return np.random.default_rng(0).integers(3, DEC_VOCAB, (DEC_SESSIONS, DEC_PROMPT)).astype(np.int32)


def decoder_config(world, per_gpu=None):
    sessions = (per_gpu or DEC_SESSIONS // world) * world
    return {"workload": f"needle2_config5_decode_{sessions}x{DEC_PROMPT}", "sessions": sessions,
            "prompt_tokens": DEC_PROMPT, "d_model": 512, "layers": 12, "heads": 8, "kv_heads": 4, "head_dim": 64,
            "vocab": DEC_VOCAB, "engram_layers": [2, 9], "matmul": "fp32 (CQ dequant-accumulate)", "kv_cache": "int8",
            "weights": "CQ4 embedding + mHC, CQ2 projections + engram tables (reference quantizer)",
            "parallelism": f"sessions split over {world} GPU(s), weights replicated, no collective",
            "l2": f"inputs larger than L2: each step reads more than {sessions * 12 * 4 * 2 * 68 * DEC_PROMPT / 1e9:.1f} GB "
                  "of INT8 KV"}


def decode_bytes(sessions, position):
    """Algorithmic HBM bytes of one decode step of `sessions` sequences whose
    new token sits at `position`: the KV cache read (position + 1 slots of
    K and V, int8 + one FP32 scale per KV head, 12 layers) and the new slot
    written, the weights once (packed CQ + FP32 tensors), the lane state
    (4 lanes x 512 FP32) read and written once per layer, the logits written
    once and read once by the greedy choice."""
    kv_slot = 4 * (2 * 64 + 2 * 4)
    kv = sessions * 12 * kv_slot * (position + 1 + 1)
    weights = 14_977_344 + 12 * (24 * 2048 * 4)    # packed CQ records + FP32 mHC projections
    lanes = sessions * 12 * 2 * 4 * 512 * 4
    logits = sessions * DEC_VOCAB * 4 * 2
    attn_only = sessions * 12 * (kv_slot * (position + 2) + 2 * 8 * 64 * 4)
    return kv + weights + lanes + logits, attn_only


def reference_decode(archive, prompt, steps, warmup=2, seconds=None):
    """The reference's own engine on the host: NativeEngine (needle2/native.py)
    on its CPU library built from its sources (oracle/_ref), all host
    threads, INT8 KV, FP32 matmuls.  Prefill one session's prompt (untimed),
    then time single-token decode steps.  Returns (tokens/s, steps, threads)."""
    from oracle import oracle as O
    if not O.ref_available():
        return None
    os.environ["NEEDLE2_NATIVE_LIBRARY"] = str(O.REF_LIB)
    os.environ.setdefault("OMP_WAIT_POLICY", "PASSIVE")
    ref_quantize()
    from needle2.native import NativeEngine
    threads = min(cpu_threads(), 256)
    e = NativeEngine(archive, threads=threads, kv_cache="int8")
    logits = e.prefill(prompt, last_only=True)
    tok = int(np.argmax(logits))
    for _ in range(warmup):
        tok = int(np.argmax(e.step(tok)))
    t0 = time.perf_counter()
    n = 0
    while True:
        tok = int(np.argmax(e.step(tok)))
        n += 1
        el = time.perf_counter() - t0
        if n >= steps or (seconds is not None and el >= seconds):
            break
    return n / el, n, threads


def run_reference_arm(args, rank, world):
    if rank != 0:
        return None
    archive = decoder_archive()
    steps = max(1, min(args.steps, 64))
    r = reference_decode(archive, decoder_prompts()[0], steps, warmup=args.warmup, seconds=120)
    if r is None:
        return {"impl": "reference", "unavailable": "the reference's CPU build (oracle/_ref) is missing"}
    tps, n, threads = r
    return {
        "impl": "reference", "metric": "batched_decode_tokens_per_s", "value": tps, "unit": "tokens/s",
        "n_gpus": world, "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 / tps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decoder_config(world),
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"{n} decode steps of one session (the reference serves one sequence per engine) "
                                   f"after its {DEC_PROMPT}-token prefill, NativeEngine on oracle/_ref with "
                                   f"{threads} threads; x86 runs the reference's portable (non-NEON) branches"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def decoder_native(args, rank, world, dist, dev):
    import torch
    from openneedle_b200.engine import GpuModel

    if DEC_SESSIONS % world:
        raise SystemExit(f"{DEC_SESSIONS} sessions do not split over {world} GPUs")
    S = args.sessions_per_gpu or DEC_SESSIONS // world
    archive = decoder_archive()
    model = GpuModel(archive, kv_cache="int8", matmul="fp32")
    batch = model.batch(S)
    prompts = np.resize(decoder_prompts(), (S * world, DEC_PROMPT))[rank * S:(rank + 1) * S]
    t0 = time.perf_counter()
    _, first = batch.prefill(prompts, logits=False, greedy=True)
    prefill_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream(dev)
    cur = torch.from_numpy(first).to(dev)
    warm = torch.empty(S, args.warmup, dtype=torch.int32, device=dev)
    batch.decode_greedy_device(cur, args.warmup, warm, stream)
    cur = warm[:, -1].contiguous()
    out = torch.empty(S, args.steps, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    position0 = int(batch.positions()[0])
    with ClockSampler(dev.index) as clocks:
        if args.profile_range:
            torch.cuda.profiler.start()
        start.record(stream)
        batch.decode_greedy_device(cur, args.steps, out, stream)
        end.record(stream)
        torch.cuda.synchronize(dev)
        if args.profile_range:
            torch.cuda.profiler.stop()
    elapsed_ms = start.elapsed_time(end)
    batch_kernels = batch.step_kernels()
    cur = out[:, -1].contiguous()

    # per-stage breakdown of a few more steps (profiled separately: events at
    # every stage boundary)
    batch.profile(True)
    prof_steps = 4
    prof_out = torch.empty(S, prof_steps, dtype=torch.int32, device=dev)
    position_p = int(batch.positions()[0])
    batch.decode_greedy_device(cur, prof_steps, prof_out, stream)
    stages = {k: v / prof_steps for k, v in batch.profile_read().items()}
    batch.profile(False)
    cur_host = prof_out[:, -1].cpu().numpy()

    # end to end through the public host-pointer call: tokens in, greedy tokens out, every step
    n_e2e = 8
    tok = cur_host
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        _, tok = batch.step(tok, logits=False, greedy=True)
    e2e_s = (time.perf_counter() - t0) / n_e2e

    t = torch.tensor([elapsed_ms, e2e_s, prefill_s], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_s, prefill_s = t.tolist()
    ms_step = elapsed_ms / args.steps
    tokens_per_s = S * world * args.steps / (elapsed_ms * 1e-3)
    mid = position0 + args.steps // 2
    step_bytes_all, _ = decode_bytes(S, mid)
    _, attn_bytes = decode_bytes(S, position_p + prof_steps // 2)
    hbm, peak_kind = peaks()
    attn_ms = stages["kv_store+attention"]
    total_prof = sum(stages.values())
    dominant = max(stages, key=stages.get)
    attn_gbs = attn_bytes / (attn_ms * 1e-3) / 1e9
    step_gbs = step_bytes_all / (ms_step * 1e-3) / 1e9
    result = {
        "metric": "batched_decode_tokens_per_s",
        "value": tokens_per_s,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": decoder_config(world, S),
        "roofline": {"bound": "hbm", "achieved": attn_gbs, "peak": hbm, "unit": "GB/s", "frac": attn_gbs / hbm,
                     "peak_source": peak_kind,
                     "kernel": "attention stage (attn_stream_kernel, one launch per layer, 12 per step; with "
                               "fewer sessions also attn_combine_rot_kernel); achieved and traffic per launch",
                     "stage_ms_per_step": attn_ms, "algorithmic_bytes_per_step": attn_bytes,
                     "algorithmic_bytes_per_launch": attn_bytes / 12,
                     "traffic": profiled_traffic("attn_stream_decode_config5")},
        "step_hbm": {"achieved_gbs": step_gbs, "frac": step_gbs / hbm, "algorithmic_bytes_per_step": step_bytes_all,
                     "note": "all of a step's algorithmic bytes (decode_bytes) over the timed step"},
        "stages_ms_per_step": stages,
        "dominant_stage": dominant,
        "profiled_step_ms": total_prof,
        "e2e": {"value": S * world / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4 * S,
                "d2h_bytes_per_step": 4 * S, "ms_per_step": e2e_s * 1e3,
                "call": "needle2_batch_step per step (this rank's sessions' tokens copied in from host memory, "
                        "their greedy tokens read back; synchronised)"},
        "prefill_s": prefill_s,
        "positions": [position0, position0 + args.steps],
        "sessions_per_gpu": S,
        "gpu_launches": batch_kernels * args.steps,
        "gpu_launches_note": "kernels of one captured decode step x K steps (the first step launches the same "
                             "kernels one by one)",
        "timing": "K decode steps in one needle2_batch_decode_greedy_device call between CUDA events on the "
                  "launching stream; max over ranks",
        "clocks": clocks.summary(),
    }
    batch.close()
    model.close()
    return result, archive


def run_native(args, rank, world, dist):
    import torch
    from openneedle_b200 import build as b

    if rank == 0:
        b.build()
    if dist is not None:
        dist.barrier()
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    result, archive = decoder_native(args, rank, world, dist, dev)
    if not args.skip_gemv:
        result["cq_gemv"] = gemv_native(args, rank, world, dist)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = reference_decode(archive, decoder_prompts()[0], 64, seconds=args.cpu_seconds)
        if r is not None:
            tps, n, threads = r
            result["cpu_baseline"] = {
                "value": tps, "unit": "tokens/s", "cores": threads, "kind": "reference",
                "sample": f"{n} decode steps of one session after its {DEC_PROMPT}-token prefill (the reference "
                          f"serves one sequence per engine), NativeEngine on oracle/_ref with {threads} threads, "
                          f"~{args.cpu_seconds:.0f} s bound; x86 runs the reference's portable branches"}
    return result


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64,
                    help="timed decode steps (config 5: 64 greedy steps)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--copies", type=int, default=0, help=f"matrices per step (default {COPIES})")
    ap.add_argument("--skip-fp32", action="store_true", help="omit the FP32-mode side measurement")
    ap.add_argument("--skip-e2e", action="store_true", help="omit the host-buffer end-to-end measurement")
    ap.add_argument("--skip-gemm", action="store_true", help="omit the prefill GEMM side measurement")
    ap.add_argument("--skip-sweep", action="store_true", help="omit the config-3 prefill GEMM shape sweep")
    ap.add_argument("--skip-attention", action="store_true", help="omit the INT8 KV attention side measurement")
    ap.add_argument("--skip-gemv", action="store_true", help="omit the fused CQ4 GEMV side line")
    ap.add_argument("--sessions-per-gpu", type=int, default=0,
                    help="decode sessions per GPU (default: config 5's 1024 split over the GPUs); other values "
                         "measure one GPU's share of a larger run and name the workload accordingly")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the timed decode steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--skip-sharded", action="store_true",
                    help="omit the N-sharded GEMM + all-gather side measurement (multi-GPU runs)")
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
            local = int(os.environ.get("LOCAL_RANK", 0))
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        try:
            result = run_native(args, rank, world, dist)
        finally:
            if dist is not None:
                dist.destroy_process_group()
    if rank == 0 and result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
