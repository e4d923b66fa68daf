#!/usr/bin/env python
"""Benchmark of the B200 matmul path: wide-MLP training samples/s.

Workload (headline): one data-parallel training step of the wide MLP
4096->4096->4096->4096->1000 (ReLU, cross-entropy with labels, momentum SGD
with clipping), global batch 8192 split by rows over N GPUs, fp32-class
arithmetic (3xTF32 tcgen05 GEMMs), synthetic seeded inputs.  A "step" is one
forward + backward + gradient all-reduce + update over the global batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0.  `value` = global samples per second with inputs
resident in HBM (max step time over ranks, CUDA events); `e2e` = the same
through the public step call with each step's batch copied from pinned host
memory and the loss read back.  `--impl reference` times the reference's CPU
implementation of the path (the NpArray restatement in oracle/, on all host
cores) on the same workload, one bounded row sample per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

DIMS = [4096, 4096, 4096, 4096, 1000]
GLOBAL_BATCH = 8192
METRIC = "MLP train samples/s (wide MLP 4096-4096-4096-4096-1000, global batch 8192)"
WORKLOAD = "wide_mlp_dp_train_step"
FLOP_PER_SAMPLE = None  # filled from DIMS below


def flops_per_sample(dims):
    fwd = sum(2 * dims[i] * dims[i + 1] for i in range(len(dims) - 1))
    dw = fwd
    dx = sum(2 * dims[i] * dims[i + 1] for i in range(1, len(dims) - 1))
    return fwd + dw + dx


FLOP_PER_SAMPLE = flops_per_sample(DIMS)
# dram__bytes_read.sum + dram__bytes_write.sum of one tc_gemm_kernel<3,1,1>
# launch (dX = dY.W^T, 8192x4096x4096) of the 1-GPU step, from one ncu capture
# of `bench.py --steps 2 --warmup 3 --skip-cpu --skip-gemm --skip-configs --no-graph`
# (algorithmic bytes of that launch: 939.5 MB).
STEP_DX_TRAFFIC_BYTES = 1748.2e6


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "sm_max_mhz": 1965.0}, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "samples": len(sm),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------- CPU baseline
def _oracle_model():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test/baseline infrastructure only
    from moonxi_net_b200 import synthetic
    threads = oracle.default_threads()
    w, b, _, _ = synthetic.mlp_problem("wide", batch=1)
    return oracle, oracle.MLPOracle(w, b, threads=threads), threads


def _rows(rng, n):
    x = rng.standard_normal((n, DIMS[0]), dtype=np.float32)
    y = rng.integers(0, DIMS[-1], n).astype(np.float32)
    return x, y


def _fit_full_step(pts):
    """Least-squares line t = fixed + rows * per_row through (rows, seconds)
    points of the CPU step; returns (fixed_s, per_row_s, full_step_s) for the
    global batch.  A step of the NpArray path has a fixed part (the
    transposed weight copies of every matmul, nparray/trait_impl.mbt:205-249,
    and the optimizer pass over all 54.4M parameters, :280-311) and a part
    linear in the rows, so a sample of a few rows must not be divided by its
    own row count."""
    r = np.array([p[0] for p in pts], np.float64)
    t = np.array([p[1] for p in pts], np.float64)
    per_row, fixed = np.polyfit(r, t, 1)
    if per_row <= 0:  # noise: fall back to the largest sample's rate
        k = int(np.argmax(r))
        per_row, fixed = t[k] / r[k], 0.0
    fixed = max(0.0, float(fixed))
    return fixed, float(per_row), fixed + GLOBAL_BATCH * float(per_row)


def _calibrate(m, rng):
    """(fixed_s, per_row_s, points) estimate of the CPU step from 8 and 40
    rows; the points also enter the final fit."""
    pts = []
    for n in (8, 40):
        x, y = _rows(rng, n)
        t0 = time.perf_counter()
        m.step(x, y, denom=GLOBAL_BATCH)
        pts.append((n, time.perf_counter() - t0))
    per_row = max((pts[1][1] - pts[0][1]) / 32.0, 1e-4)
    return max(pts[0][1] - 8 * per_row, 0.0), per_row, pts


def _sample_sizes(fixed, per_row, budget_s):
    """Two row counts for the fit: 16 and the largest multiple of 16 (<= 512)
    whose step fits `budget_s`."""
    large = int((budget_s - fixed) / per_row) // 16 * 16
    return 16, max(64, min(512, large))


def cpu_rate_sample(target_s: float):
    """Times the oracle (NpArray restatement, all host threads) on two row
    samples of the wide-MLP step and extrapolates the full 8192-row step.
    Returns the cpu_baseline dict."""
    oracle, m, threads = _oracle_model()
    rng = np.random.default_rng(3)
    fixed0, per_row0, pts = _calibrate(m, rng)
    small, large = _sample_sizes(fixed0, per_row0, max(1.0, target_s / 2 - fixed0))
    for n in (small, large):
        x, y = _rows(rng, n)
        t0 = time.perf_counter()
        m.step(x, y, denom=GLOBAL_BATCH)
        pts.append((n, time.perf_counter() - t0))
    fixed, per_row, full = _fit_full_step(pts)
    return {"value": GLOBAL_BATCH / full, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"NpArray restatement, one fwd+bwd+SGD step at {small} and {large} rows "
                      f"({pts[-2][1]:.2f} s, {pts[-1][1]:.2f} s; with the 8- and 40-row "
                      f"calibration steps, 4 points); fitted fixed {fixed:.2f} s + "
                      f"{per_row * 1e3:.2f} ms/row, extrapolated to the {GLOBAL_BATCH}-row "
                      f"step ({full:.1f} s)",
            "fixed_s": round(fixed, 3), "per_row_ms": round(per_row * 1e3, 3),
            "full_step_s": round(full, 2)}


def run_reference(args):
    """The reference's CPU algorithm (the NpArray restatement, all host
    threads) on the same workload.  Each step runs a bounded row sample of
    the global batch, alternating two sample sizes; the rate is the
    full-batch step extrapolated from the fitted fixed + per-row cost."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0  # the CPU reference runs once, on rank 0
    oracle, m, threads = _oracle_model()
    rng = np.random.default_rng(3)
    # about 90 s of sampled steps in all (the mean of the two sizes per step)
    budget_per_step = max(1.0, 90.0 / max(1, args.steps + args.warmup))
    fixed0, per_row0, cal_pts = _calibrate(m, rng)
    small, large = _sample_sizes(fixed0, per_row0, 2 * budget_per_step - fixed0 - 16 * per_row0)
    samples = {small: _rows(rng, small), large: _rows(rng, large)}
    sizes = [small if i % 2 == 0 else large for i in range(args.steps)]
    for i in range(args.warmup):
        x, y = samples[small if i % 2 == 0 else large]
        m.step(x, y, denom=GLOBAL_BATCH)
    pts = []
    t_all = time.perf_counter()
    for n in sizes:
        x, y = samples[n]
        t0 = time.perf_counter()
        m.step(x, y, denom=GLOBAL_BATCH)
        pts.append((n, time.perf_counter() - t0))
    dt = time.perf_counter() - t_all
    fixed, per_row, full = _fit_full_step(cal_pts + pts)
    value = GLOBAL_BATCH / full
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs, uniform labels, Kaiming-uniform weights)",
        "config": {"workload": WORKLOAD, "layers": DIMS, "global_batch": GLOBAL_BATCH,
                   "rows_per_step_samples": [small, large]},
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": f"each timed step is one fwd+bwd+SGD step of the NpArray "
                                   f"restatement on {small} or {large} rows (alternating; "
                                   f"with calibration steps at 8 and 40 rows in the fit); "
                                   f"fitted fixed {fixed:.2f} s + {per_row * 1e3:.2f} ms/row, "
                                   f"value = {GLOBAL_BATCH} / ({full:.1f} s extrapolated "
                                   f"{GLOBAL_BATCH}-row step); ms_per_step is the mean "
                                   f"sampled step",
                         "fixed_s": round(fixed, 3), "per_row_ms": round(per_row * 1e3, 3),
                         "full_step_s": round(full, 2)},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------- GPU
def measure_tf32_peak(torch, dev, n=8192):
    """cuBLAS TF32 GEMM throughput (TFLOP/s), best of 10: the roofline
    denominator of the TF32 tensor pipe on this GPU."""
    a = torch.randn((n, n), device=dev)
    b = torch.randn((n, n), device=dev)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for _ in range(3):
            torch.matmul(a, b)
        best = float("inf")
        for _ in range(10):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1) / 1e3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2.0 * n ** 3 / best / 1e12


def measure_cublas_sgemm(torch, dev, n=8192):
    """cuBLAS true-FP32 SGEMM throughput (TFLOP/s), median of 5 with L2
    flushed: the vendor library's figure for the exact-fp32 path, reported
    beside the SIMT kernel's as context (not part of any timed path)."""
    a = torch.randn((n, n), device=dev)
    b = torch.randn((n, n), device=dev)
    c = torch.empty((n, n), device=dev)
    flush = torch.empty(int(256e6) // 4, device=dev)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for _ in range(2):
            torch.matmul(a, b, out=c)
        times = []
        for _ in range(5):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / 1e3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c, flush
    return 2.0 * n ** 3 / statistics.median(times) / 1e12


def _time_median(torch, fn, flush, reps=5, warm=2):
    """Median CUDA-event time (s) of fn() on the current stream, L2 flushed
    (a 256 MB write) before every timed call."""
    for _ in range(warm):
        fn()
    times = []
    for _ in range(reps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    return statistics.median(times)


def gemm_sweep(torch, ops, peaks, dev, sizes=(8192,)):
    """TFLOP/s of the square NN GEMM per precision (L2 flushed between runs)."""
    out = {}
    flush = torch.empty(int(256e6) // 4, device=dev)
    for n in sizes:
        a = torch.randn((n, n), device=dev)
        b = torch.randn((n, n), device=dev)
        c = torch.empty((n, n), device=dev)
        res = {}
        for prec in ("3xtf32", "tf32", "fp32"):
            t = _time_median(torch, lambda: ops.gemm(a, b, n, n, n, out=c, precision=prec), flush)
            res[prec] = round(2.0 * n ** 3 / t / 1e12, 2)
        out[f"{n}^3_nn_tflops"] = res
        del a, b, c
    return out


def square_config_sweep(torch, ops, dev, tf32_peak, fp32_peak):
    """BASELINE config "Square fp32 GEMM sweep": M=N=K in 512..8192, NN/NT/TN,
    with and without the bias+ReLU epilogue, N(0,1) entries seed 1, every
    precision; TFLOP/s (GPU time from CUDA-graph replays, L2 flushed before
    each call; the per-call path's operand split passes included) and the
    fraction of the precision's peak (3xTF32 in TF32-equivalent terms,
    3 x 2N^3)."""
    from moonxi_net_b200 import synthetic
    flush = torch.empty(int(256e6) // 4, device=dev)
    rows = {}
    for n in (512, 1024, 2048, 4096, 8192):
        for lay, (ta, tb) in (("nn", (0, 0)), ("nt", (0, 1)), ("tn", (1, 0))):
            a_np, b_np, bias_np = synthetic.gemm_problem(n, n, n, ta, tb, 1, True)
            a = torch.from_numpy(a_np).to(dev)
            b = torch.from_numpy(b_np).to(dev)
            bias = torch.from_numpy(bias_np).to(dev)
            c = torch.empty((n, n), device=dev)
            for epi in ("plain", "bias_relu"):
                bv, relu = (bias, True) if epi == "bias_relu" else (None, False)
                for prec in ("3xtf32", "tf32", "fp32"):
                    t = _time_graph(torch, lambda: ops.gemm(a, b, n, n, n, ta=ta, tb=tb, bias=bv,
                                                            relu=relu, out=c, precision=prec),
                                    flush, reps=10 if n <= 2048 else 3)
                    tf = 2.0 * n ** 3 / t / 1e12
                    frac = (3 * tf / tf32_peak if prec == "3xtf32" else
                            tf / tf32_peak if prec == "tf32" else tf / fp32_peak)
                    rows[f"{n}_{lay}_{epi}_{prec}"] = [round(tf, 2), round(frac, 3)]
            del a, b, c, bias
    return {"unit": "[TFLOP/s, fraction of peak]", "peaks_tflops": {
        "tf32": round(tf32_peak, 1), "fp32_simt": round(fp32_peak, 1)}, "results": rows}


def _time_graph(torch, fn, flush, reps=10):
    """GPU time (s) of one fn() call, host launch overhead excluded: fn is
    captured in a CUDA graph after an L2 flush (a 256 MB write), R times; the
    same graph without fn is timed too and subtracted."""
    fn()  # sizes any workspace before capture
    torch.cuda.synchronize()
    graphs = []
    for with_fn in (True, False):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                flush.zero_()
                if with_fn:
                    fn()
        graphs.append(g)
    best = []
    for g in graphs:
        g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(3):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 1e3)
        best.append(statistics.median(ts))
    return max(best[0] - best[1], 1e-9) / reps


def ragged_config_sweep(torch, ops, dev, hbm_peak, tf32_peak, fp32_peak):
    """BASELINE config "Ragged/skinny GEMMs": M in {1,7,33,127,1000} x K in
    {512,784,3072,4096} x N in {10,100,257,1000}, N(0,1) seed 4, NN/NT/TN,
    bias+ReLU epilogue, the default (AUTO) precision.  M <= 33 is judged on
    HBM bandwidth (algorithmic bytes 4(MK+KN+MN+N)), the others on TFLOP/s.
    GPU time per call from CUDA-graph replays with L2 flushed before each
    call (host launch overhead excluded; it dominates the smallest shapes)."""
    from moonxi_net_b200 import synthetic
    flush = torch.empty(int(256e6) // 4, device=dev)
    per_m = {}
    for M in (1, 7, 33, 127, 1000):
        vals = []
        for K in (512, 784, 3072, 4096):
            for N in (10, 100, 257, 1000):
                for ta, tb in ((0, 0), (0, 1), (1, 0)):
                    a_np, b_np, bias_np = synthetic.gemm_problem(M, K, N, ta, tb, 4, True)
                    a = torch.from_numpy(a_np).to(dev)
                    b = torch.from_numpy(b_np).to(dev)
                    bias = torch.from_numpy(bias_np).to(dev)
                    c = torch.empty((M, N), device=dev)
                    t = _time_graph(torch, lambda: ops.gemm(a, b, M, K, N, ta=ta, tb=tb,
                                                            bias=bias, relu=True, out=c),
                                    flush)
                    if M <= 33:
                        vals.append(4.0 * (M * K + K * N + M * N + N) / t / 1e9)
                    else:
                        vals.append(2.0 * M * N * K / t / 1e12)
        vals.sort()
        if M <= 33:
            per_m[f"M={M}"] = {"unit": "GB/s", "median": round(statistics.median(vals), 1),
                               "min": round(vals[0], 1), "max": round(vals[-1], 1),
                               "median_frac_of_hbm": round(statistics.median(vals) / hbm_peak, 3),
                               "shapes": len(vals)}
        else:
            per_m[f"M={M}"] = {"unit": "TFLOP/s", "median": round(statistics.median(vals), 2),
                               "min": round(vals[0], 2), "max": round(vals[-1], 2),
                               "median_frac_of_fp32_simt": round(statistics.median(vals) /
                                                                 fp32_peak, 3),
                               "shapes": len(vals)}
    return {"hbm_peak_gbs": hbm_peak, "precision": "auto (exact FP32 SIMT for these shapes "
            "unless M, N >= 128 and 2MNK >= 1e9: 3xTF32)", "per_M": per_m}


def mlp_config_bench(torch, nn, synthetic, dev, tf32_peak):
    """BASELINE configs "MLP 3072->1024->1024->10, batch 512, 200 steps"
    (samples/s over 200 captured steps) and "MLP 784->256->10, batch 64"
    (latency of one captured step), both 3xTF32 on one GPU."""
    out = {}
    for name, dims, batch, steps in (("mlp3072", [3072, 1024, 1024, 10], 512, 200),
                                     ("mlp784", [784, 256, 10], 64, 200)):
        w, b, x, y = synthetic.mlp_problem(name, batch=batch)
        m = nn.MLP(dims, w, b, precision="3xtf32")
        X, Y = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
        m.step(X, Y)
        torch.cuda.synchronize()
        m.capture(X, Y)
        for _ in range(5):
            m.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            m.replay()
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3 / steps
        fl = flops_per_sample(dims) * batch
        out[name] = {"samples_per_s": round(batch / t, 1), "ms_per_step": round(t * 1e3, 4),
                     "steps": steps, "batch": batch, "model_tflops": round(fl / t / 1e12, 2),
                     "frac_of_tf32_peak_3x": round(3 * fl / t / 1e12 / tf32_peak, 3),
                     "final_loss": float(m.loss_slot.item())}
        m.close()
        del m
    return out


def single_gpu_loss(torch, nn, synthetic, dev, n_steps):
    """Loss after n_steps of the same training on one GPU and the whole
    global batch: the reference point of a data-parallel run's loss."""
    w, b, x, y = synthetic.mlp_problem("wide")
    m = nn.MLP(DIMS, w, b, layout="nn", precision="3xtf32")
    X, Y = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
    del w, b, x, y
    for _ in range(n_steps):
        m.step(X, Y, GLOBAL_BATCH)
    loss = float(m.loss_slot.item())
    m.close()
    del m, X, Y
    torch.cuda.empty_cache()
    return loss


def run_ours(args):
    import torch
    import torch.distributed as dist

    from moonxi_net_b200 import _lib, nn, ops, synthetic

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: WORLD_SIZE={world} but --gpus={args.gpus}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        pg = dist.group.WORLD
    peaks, peak_kind = load_peaks()

    B = GLOBAL_BATCH // world
    w, b, x_all, y_all = synthetic.mlp_problem("wide")
    x_np = np.ascontiguousarray(x_all[rank * B:(rank + 1) * B])
    y_np = np.ascontiguousarray(y_all[rank * B:(rank + 1) * B])
    model = nn.MLP(DIMS, w, b, layout="nn", precision=args.precision, process_group=pg,
                   shard_update=args.shard_update)
    del w, b, x_all, y_all
    X = torch.from_numpy(x_np).to(dev)
    Y = torch.from_numpy(y_np).to(dev)
    x_pin = torch.from_numpy(x_np).pin_memory()
    y_pin = torch.from_numpy(y_np).pin_memory()

    def barrier():
        if pg is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # eager warm-up sizes every workspace; then capture the step
    model.step(X, Y, GLOBAL_BATCH)
    torch.cuda.synchronize()
    use_graph = not args.no_graph
    launches_per_step = None
    if use_graph:
        n0 = _lib.lib().mx_kernel_launch_count()
        model.capture(X, Y, GLOBAL_BATCH)
        launches_per_step = _lib.lib().mx_kernel_launch_count() - n0
        run_step = model.replay
    else:
        def run_step():
            return model.step(X, Y, GLOBAL_BATCH)
    for _ in range(args.warmup):
        run_step()
    barrier()

    # ---- timed region: inputs resident in HBM
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    n_launch0 = _lib.lib().mx_kernel_launch_count()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record()
    for _ in range(args.steps):
        run_step()
    e1.record()
    barrier()
    clk = clocks.stop()
    elapsed = e0.elapsed_time(e1) / 1e3
    if not use_graph:
        launches_per_step = (_lib.lib().mx_kernel_launch_count() - n_launch0) / args.steps
    t = torch.tensor([elapsed], device=dev)
    if pg is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed = float(t.item())
    value = GLOBAL_BATCH * args.steps / elapsed

    # ---- e2e: every step copies its batch from pinned host memory and reads
    # the loss back, through the library's HostBatchPipeline: the next batch
    # is uploaded on a copy stream while the current step runs (two input
    # buffers, one captured step per buffer); the timed region holds every
    # copy and read.
    if use_graph:
        model.release_graph()
    pipe = nn.HostBatchPipeline(model, B, GLOBAL_BATCH, use_graph=use_graph)
    barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record()
    loss_host = pipe.run([(x_pin, y_pin)] * args.steps)
    e3.record()
    barrier()
    e2e_t = torch.tensor([e2.elapsed_time(e3) / 1e3], device=dev)
    if pg is not None:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = GLOBAL_BATCH * args.steps / float(e2e_t.item())
    h2d = x_pin.numel() * 4 + y_pin.numel() * 4
    pipe.release()  # graphs holding NCCL calls go before the process group does
    del pipe

    # ---- GEMM time inside one eager step (roofline of the dominant kernel)
    gemm_log = []
    model.gemm_timer = gemm_log
    barrier()
    model.step(X, Y, GLOBAL_BATCH)
    barrier()
    model.gemm_timer = None
    g_flops = sum(f for f, _, _ in gemm_log)
    g_time = sum(a.elapsed_time(b_) / 1e3 for _, a, b_ in gemm_log)
    step_gpu_time = elapsed / args.steps
    # phase boundaries of one more eager step (CUDA events on the step's stream)
    marks = []
    model.phase_marks = marks
    barrier()
    model.step(X, Y, GLOBAL_BATCH)
    barrier()
    model.phase_marks = None
    phases = {marks[i][0]: round(marks[i - 1][1].elapsed_time(marks[i][1]), 3)
              for i in range(1, len(marks))}

    # ---- data-parallel correctness, outside every timed region: every
    # replica must hold bit-identical parameters (element-wise MAX == MIN over
    # the ranks), and the loss must match one GPU trained the same way
    dp_check = {}
    if pg is not None:
        model.sync_params()
        pmax = model.params.clone()
        pmin = model.params.clone()
        dist.all_reduce(pmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(pmin, op=dist.ReduceOp.MIN)
        dp_check["replicas_identical"] = bool(torch.equal(pmax, pmin))
        del pmax, pmin
        # steps so far: 1 eager + W warm-up + K timed + K e2e + 2 instrumented
        n_done = 1 + args.warmup + 2 * args.steps + 2
        if rank == 0:
            dp_loss = float(model.loss_slot.item())
            ref_loss = single_gpu_loss(torch, nn, synthetic, dev, n_done)
            dp_check.update({"steps_compared": n_done, "loss_dp": dp_loss, "loss_n1": ref_loss,
                             "loss_vs_n1": abs(dp_loss - ref_loss)})
        dist.barrier()

    # Roofline denominator of the TF32 tensor pipe: half the measured dense
    # bf16 rate of MEASURED_PEAKS.json (B200's TF32 rate is half its bf16
    # rate), the burst figure.  A cuBLAS TF32 GEMM measured in this run is
    # reported beside it as context.  A 3xTF32 GEMM issues three TF32 MMAs
    # per algorithmic multiply-add.
    tf32_peak = peaks["bf16_tflops"] / 2.0
    tf32_peak_sustained = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) / 2.0
    tf32_cublas = measure_tf32_peak(torch, dev)
    # FP32 SIMT peak: 148 SMs x 128 FP32 lanes x 2 FLOP x max SM clock
    fp32_peak = 148 * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
    achieved_tc = 3.0 * g_flops / g_time / 1e12 if g_time > 0 else 0.0

    gemm_bench = {}
    configs = {}
    if rank == 0 and world == 1 and not args.skip_gemm:
        gemm_bench = gemm_sweep(torch, ops, peaks, dev)
        r = gemm_bench["8192^3_nn_tflops"]
        gemm_bench["frac_of_peak"] = {
            "3xtf32_tf32_equivalent": round(3.0 * r["3xtf32"] / tf32_peak, 3),
            "tf32": round(r["tf32"] / tf32_peak, 3),
            "fp32_simt": round(r["fp32"] / fp32_peak, 3)}
        gemm_bench["peaks_tflops"] = {
            f"tf32_{peak_kind}_bf16_half": round(tf32_peak, 1),
            "tf32_cublas_this_run": round(tf32_cublas, 1),
            "fp32_simt_nominal_at_max_clock": round(fp32_peak, 1)}
        sgemm = measure_cublas_sgemm(torch, dev)
        gemm_bench["cublas_sgemm_8192_tflops"] = round(sgemm, 2)
        gemm_bench["fp32_simt_vs_cublas_sgemm"] = round(r["fp32"] / sgemm, 3)
    if rank == 0 and world == 1 and not args.skip_configs:
        configs["square_sweep"] = square_config_sweep(torch, ops, dev, tf32_peak, fp32_peak)
        configs["ragged"] = ragged_config_sweep(torch, ops, dev, peaks["hbm_gbs"], tf32_peak,
                                                fp32_peak)
        configs.update(mlp_config_bench(torch, nn, synthetic, dev, tf32_peak))

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_rate_sample(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * elapsed / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) inputs, uniform labels, Kaiming-uniform weights)",
            "config": {"workload": WORKLOAD, "layers": DIMS, "global_batch": GLOBAL_BATCH,
                       "per_gpu_batch": B, "precision": args.precision,
                       "parallelism": f"dp{world}", "cuda_graph": use_graph,
                       "optimizer_update": "sharded (reduce-scatter / all-gather)"
                       if model.sharded else ("replicated (all-reduce)" if world > 1
                                              else "single GPU"),
                       "l2": "inputs larger than L2 (217.8 MB of weights + 128 MB batch "
                             "per step), no explicit flush"},
            "roofline": {"bound": "tensor", "achieved": round(achieved_tc, 1),
                         "peak": round(tf32_peak, 1), "unit": "TFLOP/s",
                         "frac": round(achieved_tc / tf32_peak, 4),
                         "frac_of_sustained": round(achieved_tc / tf32_peak_sustained, 4),
                         "tf32_cublas_this_run": round(tf32_cublas, 1),
                         "traffic": STEP_DX_TRAFFIC_BYTES if B == GLOBAL_BATCH else None,
                         "traffic_note": "DRAM read+write bytes of one dX launch "
                                         "(8192x4096x4096) from an ncu capture of this "
                                         "step; algorithmic 939.5 MB",
                         "kernel": "tc_gemm_kernel<3> (tcgen05 kind::tf32, 3 MMAs per "
                                   "multiply-add), TF32 tensor FLOP = 3 x 2MNK",
                         "peak_source": f"MEASURED_PEAKS.json bf16_tflops / 2 ({peak_kind}, "
                                        "burst); frac_of_sustained uses "
                                        "bf16_tflops_sustained / 2",
                         "gemm_share_of_step": round(g_time / step_gpu_time, 3)
                         if step_gpu_time > 0 else None,
                         "algorithmic_tflops": round(g_flops / g_time / 1e12, 1)
                         if g_time > 0 else None},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "samples/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk,
            "gemm": gemm_bench,
            "configs": configs,
            "dp_check": dp_check,
            "flop_per_sample": FLOP_PER_SAMPLE,
            "model_tflops": round(value * FLOP_PER_SAMPLE / 1e12, 1),
            "final_loss": loss_host[-1] if loss_host else None,
            "step_phases_ms_rank0_eager": phases,
        }
        print(json.dumps(line), flush=True)
    model.close()  # its NCCL communicator (every rank), before the process group
    if pg is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_gemm_only(args):
    """One GEMM (square N^3 with --gemm N, or --shape M,K,N), K timed launches
    after W warm-ups (L2 flushed between launches); the small cases the kernel
    profiles are taken on."""
    import torch

    from moonxi_net_b200 import ops
    torch.cuda.set_device(0)
    if args.shape:
        M, K, N = (int(v) for v in args.shape.split(","))
    else:
        M = K = N = args.gemm
    ta, tb = {"nn": (0, 0), "nt": (0, 1), "tn": (1, 0)}[args.layout]
    a = torch.randn((K, M) if ta else (M, K), device="cuda")
    b = torch.randn((N, K) if tb else (K, N), device="cuda")
    c = torch.empty((M, N), device="cuda")
    flush = torch.empty(int(256e6) // 4, device="cuda")
    prec = ("3xtf32" if not args.shape else "auto") if args.precision == "auto" else args.precision
    for _ in range(args.warmup):
        ops.gemm(a, b, M, K, N, ta=ta, tb=tb, out=c, precision=prec)
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.gemm(a, b, M, K, N, ta=ta, tb=tb, out=c, precision=prec)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    t = statistics.median(times)
    by = 4.0 * (M * K + K * N + M * N)
    print(json.dumps({"metric": f"GEMM {M}x{K}x{N} {args.layout}", "precision": prec,
                      "tflops": 2.0 * M * N * K / t / 1e12, "gbs": by / t / 1e9, "ms": t * 1e3,
                      "steps": args.steps, "warmup": args.warmup}), flush=True)
    return 0


def run_pair_only(args):
    """One Linear layer's backward (layout nn: dX = dY W^T masked, with split
    output and column sums; dW = X^T dY) through mx_gemm_split_pair, K timed
    calls after W warm-ups (L2 flushed between calls); --pair B,FI,FO, with
    --sm-budget S preferring S SMs as a data-parallel step does."""
    import torch

    from moonxi_net_b200 import ops
    torch.cuda.set_device(0)
    B, fi, fo = (int(v) for v in args.pair.split(","))
    ctx = ops.new_context(0)
    if args.sm_budget:
        ops.set_sm_budget(ctx, args.sm_budget)

    def split(rows, cols):
        x = torch.randn(rows, cols, device="cuda")
        hi = torch.empty(rows * cols + 64, device="cuda")
        lo = torch.empty(rows * cols + 64, device="cuda")
        ops.split_tf32(x, hi[:rows * cols].view(rows, cols), lo[:rows * cols].view(rows, cols),
                       ctx=ctx)
        return x, hi, lo
    _, gh, gl = split(B, fo)       # dY
    h, hh, hl = split(B, fi)       # layer input (its ReLU mask)
    _, wh, wl = split(fi, fo)      # W [in, out]
    dx, dx_hi, dx_lo = (torch.empty(B * fi, device="cuda") for _ in range(3))
    dw = torch.empty(fi * fo, device="cuda")
    cs = torch.empty(fi, device="cuda")
    scratch = torch.empty(ops.gemm_colsum_scratch_bytes(B, fi) // 4, device="cuda")
    dx_kw = dict(a_hi=gh, a_lo=gl, lda=fo, a_kmajor=True, b_hi=wh, b_lo=wl, ldb=fo,
                 b_kmajor=True, M=B, K=fo, N=fi, c=dx, c_hi=dx_hi, c_lo=dx_lo, mask=h, ldm=fi,
                 colsum=cs, colsum_scratch=scratch, padded=3)
    dw_kw = dict(a_hi=hh, a_lo=hl, lda=fi, a_kmajor=False, b_hi=gh, b_lo=gl, ldb=fo,
                 b_kmajor=False, M=fi, K=B, N=fo, c=dw, padded=3)
    flush = torch.empty(int(256e6) // 4, device="cuda")
    for _ in range(args.warmup):
        ops.gemm_split_pair(dx_kw, dw_kw, ctx=ctx)
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.gemm_split_pair(dx_kw, dw_kw, ctx=ctx)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    rc, where = ops.context_status(ctx)
    ops.destroy_context(ctx)
    if rc != 0:
        print(f"status {rc} at call site {where}", file=sys.stderr)
        return 1
    t = statistics.median(times)
    fl = 2.0 * 2 * B * fi * fo
    print(json.dumps({"metric": f"layer backward pair B={B} {fi}->{fo}", "ms": t * 1e3,
                      "tflops": fl / t / 1e12, "tf32_tflops_3x": 3 * fl / t / 1e12,
                      "sm_budget": args.sm_budget, "steps": args.steps,
                      "warmup": args.warmup}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "fp32", "tf32", "auto"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--shard-update", dest="shard_update", action="store_const", const=True,
                    default=None,
                    help="N>1: reduce-scatter the gradients, update 1/N of the parameters "
                         "per rank, all-gather the weights (the model's default from 4 GPUs)")
    ap.add_argument("--replicated-update", dest="shard_update", action="store_const",
                    const=False,
                    help="N>1: all-reduce the gradients and update every parameter on every "
                         "rank (the model's default on 2 GPUs)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-gemm", action="store_true")
    ap.add_argument("--skip-configs", action="store_true",
                    help="skip the other BASELINE configs (square sweep, ragged set, MLP "
                         "3072 and 784)")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--gemm", type=int, default=0, metavar="N",
                    help="time only the square N^3 GEMM of --precision (profiling case)")
    ap.add_argument("--layout", default="nn", choices=["nn", "nt", "tn"])
    ap.add_argument("--shape", default="", metavar="M,K,N",
                    help="time only this GEMM (any shape; default precision auto)")
    ap.add_argument("--pair", default="", metavar="B,FI,FO",
                    help="time only one Linear layer's paired backward GEMMs")
    ap.add_argument("--sm-budget", type=int, default=0,
                    help="with --pair: SMs the GEMMs prefer (a data-parallel step's 128)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 warm-up steps
    if args.impl == "reference":
        return run_reference(args)
    if args.pair:
        return run_pair_only(args)
    if args.gemm or args.shape:
        return run_gemm_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
