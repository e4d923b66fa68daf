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
# of `bench.py --steps 2 --warmup 3 --skip-cpu --skip-gemm --no-graph`
# (algorithmic bytes of that launch: 939.5 MB).
STEP_DX_TRAFFIC_BYTES = 1749.6e6


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
def cpu_rate_sample(target_s: float, dims=DIMS, max_rows: int = 256):
    """Times the oracle (NpArray restatement, all host threads) on a row
    sample of the wide-MLP step.  Returns (samples/s, rows, seconds, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test/baseline infrastructure only
    from moonxi_net_b200 import synthetic
    threads = oracle.default_threads()
    w, b, _, _ = synthetic.mlp_problem("wide", batch=1)
    rng = np.random.default_rng(3)
    # calibrate on 8 rows, then size the sample for ~target_s
    m = oracle.MLPOracle(w, b, threads=threads)
    x8 = rng.standard_normal((8, dims[0]), dtype=np.float32)
    y8 = rng.integers(0, dims[-1], 8).astype(np.float32)
    t0 = time.perf_counter()
    m.step(x8, y8)
    t_cal = time.perf_counter() - t0
    rows = int(max(8, min(max_rows, 8 * target_s / max(t_cal, 1e-3))))
    rows = max(8, rows // 8 * 8)
    x = rng.standard_normal((rows, dims[0]), dtype=np.float32)
    y = rng.integers(0, dims[-1], rows).astype(np.float32)
    t0 = time.perf_counter()
    m.step(x, y, denom=GLOBAL_BATCH)
    dt = time.perf_counter() - t0
    return rows / dt, rows, dt, threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0  # the CPU reference runs once, on rank 0
    budget_per_step = max(1.0, 90.0 / max(1, args.steps + args.warmup))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from moonxi_net_b200 import synthetic
    threads = oracle.default_threads()
    w, b, _, _ = synthetic.mlp_problem("wide", batch=1)
    m = oracle.MLPOracle(w, b, threads=threads)
    rng = np.random.default_rng(3)
    # calibrate rows per step
    x8 = rng.standard_normal((8, DIMS[0]), dtype=np.float32)
    y8 = rng.integers(0, DIMS[-1], 8).astype(np.float32)
    t0 = time.perf_counter()
    m.step(x8, y8, denom=GLOBAL_BATCH)
    t_cal = time.perf_counter() - t0
    rows = int(max(8, min(512, 8 * budget_per_step / max(t_cal, 1e-3)))) // 8 * 8
    x = rng.standard_normal((rows, DIMS[0]), dtype=np.float32)
    y = rng.integers(0, DIMS[-1], rows).astype(np.float32)
    for _ in range(args.warmup):
        m.step(x, y, denom=GLOBAL_BATCH)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.step(x, y, denom=GLOBAL_BATCH)
    dt = time.perf_counter() - t0
    value = rows * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) inputs, uniform labels, Kaiming-uniform weights)",
        "config": {"workload": WORKLOAD, "layers": DIMS, "global_batch": GLOBAL_BATCH,
                   "rows_per_step_sample": rows},
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} rows of the global batch per step (one fwd+bwd+SGD "
                                   f"over the full 54.4M-parameter model), {args.steps} steps"},
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
            for _ in range(2):
                ops.gemm(a, b, n, n, n, out=c, precision=prec)
            times = []
            for _ in range(5):
                flush.zero_()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                ops.gemm(a, b, n, n, n, out=c, precision=prec)
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) / 1e3)
            t = statistics.median(times)
            res[prec] = round(2.0 * n ** 3 / t / 1e12, 2)
        out[f"{n}^3_nn_tflops"] = res
        del a, b, c
    return out


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

    gemm_bench = {}
    if rank == 0 and world == 1 and not args.skip_gemm:
        gemm_bench = gemm_sweep(torch, ops, peaks, dev)

    # The TF32 tensor peak is measured here the way the driver measures the
    # bf16 one: a cuBLAS GEMM (torch.matmul with TF32 enabled), 8192^3, best of
    # 10, on this GPU -- a library denominator, not part of the timed path.
    # A 3xTF32 GEMM issues three TF32 MMAs per algorithmic multiply-add.
    tf32_peak = measure_tf32_peak(torch, dev)
    achieved_tc = 3.0 * g_flops / g_time / 1e12 if g_time > 0 else 0.0
    if gemm_bench:
        # FP32 SIMT peak: 148 SMs x 128 FP32 lanes x 2 FLOP x max SM clock
        fp32_peak = 148 * 128 * 2 * peaks.get("sm_max_mhz", 1965.0) * 1e6 / 1e12
        r = gemm_bench["8192^3_nn_tflops"]
        gemm_bench["frac_of_peak"] = {
            "3xtf32_tf32_equivalent": round(3.0 * r["3xtf32"] / tf32_peak, 3),
            "tf32": round(r["tf32"] / tf32_peak, 3),
            "fp32_simt": round(r["fp32"] / fp32_peak, 3)}
        gemm_bench["peaks_tflops"] = {"tf32_cublas_measured": round(tf32_peak, 1),
                                      "fp32_simt_nominal_at_max_clock": round(fp32_peak, 1)}
        sgemm = measure_cublas_sgemm(torch, dev)
        gemm_bench["cublas_sgemm_8192_tflops"] = round(sgemm, 2)
        gemm_bench["fp32_simt_vs_cublas_sgemm"] = round(r["fp32"] / sgemm, 3)

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        rate, rows, dt, threads = cpu_rate_sample(args.cpu_seconds)
        cpu = {"value": rate, "unit": "samples/s", "cores": threads, "kind": "port",
               "sample": f"{rows} rows of the global batch through one full fwd+bwd+SGD step "
                         f"of the NpArray restatement ({dt:.1f} s)"}

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
                         "traffic": STEP_DX_TRAFFIC_BYTES if B == GLOBAL_BATCH else None,
                         "traffic_note": "DRAM read+write bytes of one dX launch "
                                         "(8192x4096x4096) from an ncu capture of this "
                                         "step; algorithmic 939.5 MB",
                         "kernel": "tc_gemm_kernel<3> (tcgen05 kind::tf32, 3 MMAs per "
                                   "multiply-add), TF32 tensor FLOP = 3 x 2MNK",
                         "peak_source": "cuBLAS TF32 GEMM 8192^3 measured in this run (best "
                                        "of 10); for reference "
                                        f"{peak_kind} bf16_tflops/2 = "
                                        f"{peaks['bf16_tflops'] / 2.0:.1f}",
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
            "flop_per_sample": FLOP_PER_SAMPLE,
            "model_tflops": round(value * FLOP_PER_SAMPLE / 1e12, 1),
            "final_loss": loss_host[-1] if loss_host else None,
            "step_phases_ms_rank0_eager": phases,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_gemm_only(args):
    """One square GEMM, K timed launches after W warm-ups (L2 flushed between
    launches); the small case the kernel profiles are taken on."""
    import torch

    from moonxi_net_b200 import ops
    torch.cuda.set_device(0)
    n = args.gemm
    ta, tb = {"nn": (0, 0), "nt": (0, 1), "tn": (1, 0)}[args.layout]
    a = torch.randn((n, n), device="cuda")
    b = torch.randn((n, n), device="cuda")
    c = torch.empty((n, n), device="cuda")
    flush = torch.empty(int(256e6) // 4, device="cuda")
    prec = "3xtf32" if args.precision == "auto" else args.precision
    for _ in range(args.warmup):
        ops.gemm(a, b, n, n, n, ta=ta, tb=tb, out=c, precision=prec)
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.gemm(a, b, n, n, n, ta=ta, tb=tb, out=c, precision=prec)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / 1e3)
    t = statistics.median(times)
    print(json.dumps({"metric": f"GEMM {n}^3 {args.layout} TFLOP/s", "precision": prec,
                      "value": 2.0 * n ** 3 / t / 1e12, "unit": "TFLOP/s", "ms": t * 1e3,
                      "steps": args.steps, "warmup": args.warmup}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--precision", default="3xtf32", choices=["3xtf32", "fp32", "tf32", "auto"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--shard-update", action="store_true",
                    help="N>1: reduce-scatter the gradients, update 1/N of the parameters "
                         "per rank, all-gather the weights (default: all-reduce, replicated "
                         "update)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-gemm", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--gemm", type=int, default=0, metavar="N",
                    help="time only the square N^3 GEMM of --precision (profiling case)")
    ap.add_argument("--layout", default="nn", choices=["nn", "nt", "tn"])
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # timing rule: at least 3 warm-up steps
    if args.impl == "reference":
        return run_reference(args)
    if args.gemm:
        return run_gemm_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
