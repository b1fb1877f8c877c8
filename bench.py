#!/usr/bin/env python
"""Benchmark of the fp32-input GEMM family on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one call of the operator on one batch of synthetic input.  The
headline workload is the batched config (128 x (512x1024 . 1024x2048),
reference PID 3): every rank runs the full config on its own GPU (the batch
shards with no communication), so per-GPU work is fixed as N grows
("scaling": "weak") and `value` is the whole job's TFLOP/s.

Rank 0 prints one JSON line.  `value` is measured with inputs resident in
HBM; `e2e` is the same metric through the public API with the inputs copied
from pinned host memory and the result copied back inside the timed region.
At N=1 a per-shape table (`shapes`) covers every other config: our kernel,
cuBLAS (TF32) and the reference's own kernel side by side.

--impl reference runs the reference's own CUDA kernel for the workload
(kernels/3_Batched_matrix_multiplication_best_kernel.cu:113, compiled
unmodified for sm_100a into oracle/_ref) through its own entry point, on
every rank, timed the same way.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
PKG = "cupilot-kernels_b200"
METRIC = "GEMM TFLOP/s and % of B200 TF32 peak per shape at 1/2/4/8 GPUs"
HEADLINE = "batched"


def _pkg(sub):
    return importlib.import_module(f"{PKG}.{sub}")


# ---------------------------------------------------------------- peaks
def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "tf32_tflops": d["bf16_tflops"] / 2.0, "source": "measured",
                "tf32_note": "MEASURED_PEAKS.json bf16_tflops (cuBLAS burst) / 2: tcgen05 "
                             "kind::tf32 issues at half the kind::f16 rate"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "tf32_tflops": 795.0,
            "source": "fallback", "tf32_note": "fallback bf16 figure / 2"}


def load_traffic():
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        mhz = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        load = [m for m in mhz if m > 300] or mhz
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows
                                    if r[3].replace(".", "").isdigit()), default=None)}


# ---------------------------------------------------------------- distributed
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- timing helpers
def time_loop(fn, steps, warmup, world=1, per_launch=True):
    """Device time of `steps` calls (ms, max over ranks) and the mean per-call
    event duration, both on the current stream."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)] if per_launch else []
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(steps):
        if per_launch:
            evs[i][0].record(stream)
        fn()
        if per_launch:
            evs[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    total = max_over_ranks(t0.elapsed_time(t1), world)
    launch = statistics.mean(a.elapsed_time(b) for a, b in evs) if per_launch else None
    return total, launch


def adaptive_steps(fn, target_s=0.25, lo=5, hi=2000):
    torch.cuda.synchronize()
    t = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    dt = max(time.perf_counter() - t, 1e-5)
    return int(min(hi, max(lo, target_s / dt)))


# ---------------------------------------------------------------- workloads on device
def device_inputs(w, seed_offset=0, **shapes):
    return _pkg("workloads").device_inputs(w, seed_offset, **shapes)


def cublas_fn(name, A, B, *rest):
    """The same math through torch (cuBLAS TF32) for the comparison column."""
    if name == "pointwise_conv":   # cuDNN conv2d (TF32 allowed by default)
        return lambda: torch.nn.functional.conv2d(A, B, rest[0])
    if name == "sdpa":             # torch's fused attention (backend of its choice)
        return lambda: torch.nn.functional.scaled_dot_product_attention(A, B, rest[0])
    if name == "transposed_a":
        return lambda: torch.matmul(A.t(), B)
    if name == "transposed_b":
        return lambda: torch.matmul(A, B.t())
    if name == "transposed_both":
        return lambda: torch.matmul(A.t(), B.t())
    if name == "diag":
        return lambda: A[:, None] * B
    if name == "matrix_scalar":
        return lambda: A * B
    if name == "upper_tri":
        return lambda: torch.triu(torch.matmul(A, B))
    if name == "lower_tri":
        return lambda: torch.tril(torch.matmul(A, B))
    return lambda: torch.matmul(A, B)


def roofline(w, ms, peaks, flops=None, nbytes=None):
    # Triangular operators are measured on the flops of their non-zero band.
    flops = (w.useful_flops or w.flops) if flops is None else flops
    nbytes = w.min_bytes if nbytes is None else nbytes
    s = ms / 1e3
    tflops = flops / s / 1e12
    gbs = nbytes / s / 1e9
    # fp16 operands (attention) run at the f16 tensor rate, the rest at TF32's.
    tpeak = peaks["bf16_tflops"] if w.name == "sdpa" else peaks["tf32_tflops"]
    t_c = flops / (tpeak * 1e12)
    t_m = nbytes / (peaks["hbm_gbs"] * 1e9)
    if w.bound == "hbm" or t_m > t_c:
        return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4), "tflops": round(tflops, 2)}
    return {"bound": "tensor", "achieved": round(tflops, 2), "peak": round(tpeak, 1),
            "unit": "TFLOP/s", "frac": round(tflops / tpeak, 4),
            "gbs": round(gbs, 1)}


# ---------------------------------------------------------------- reference kernels
REF_SAFE = {  # workload -> reference PID whose kernel runs on the workload
    "matrix_scalar": 5,
    "square": 1, "batched": 3, "large_k": 6, "small_k": 7, "irregular": 8, "tall_skinny": 9,
    "tensor3d": 10, "tensor4d": 11, "diag": 12, "symmetric": 13, "upper_tri": 14,
    "lower_tri": 15, "transposed_a": 16, "transposed_b": 17, "transposed_both": 18,
    "pointwise_conv": 87, "sdpa": 97,
}


def reference_callable(name, A, B, *rest):
    from oracle import build_ref

    if name == "gemv":
        # K4 raised an illegal memory access on its first golden-vector call
        # on this GPU type (kernels/4_...:84); it is not run again.
        raise RuntimeError("reference K4 (gemv_cuda) faulted on a B200 and is not run")
    pid = REF_SAFE[name]
    f = build_ref.load(pid)
    if name == "small_k":
        # K7 reads 64 K-columns whatever K is (kernels/7_...:27-44); run it on
        # the mathematically identical zero-padded K = 64 inputs.
        Ap = torch.nn.functional.pad(A, (0, 64 - A.shape[1]))
        Bp = torch.nn.functional.pad(B, (0, 0, 0, 64 - B.shape[0]))
        return (lambda: f(Ap, Bp)), "zero-padded to K=64 (K7's own contract)"
    if name == "tall_skinny":
        return (lambda: f(A, B)), "as is; K9 uses only 32 of the 64 inner columns (parity FAIL)"
    if name == "pointwise_conv":
        return (lambda: f(A, B, rest[0])), "float32 dispatch only (its double instance fails ptxas)"
    if name == "sdpa":
        return (lambda: f(A, B, rest[0])), None
    return (lambda: f(A, B)), None


# ---------------------------------------------------------------- CPU baseline
def cpu_baseline(w, budget_s=12.0):
    """torch.matmul fp32 on the host cores over a bounded sample of the workload."""
    threads = torch.get_num_threads()
    g = torch.Generator().manual_seed(w.seed)
    sub = 16
    s = w.shapes
    A = torch.randn(sub, s["m"], s["k"], generator=g)
    B = torch.randn(sub, s["k"], s["n"], generator=g)
    flops = 2.0 * sub * s["m"] * s["n"] * s["k"]
    torch.matmul(A, B)
    reps, t0 = 0, time.perf_counter()
    while True:
        torch.matmul(A, B)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 2000:
            break
    return {"value": round(flops * reps / el / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "sample": f"torch.matmul fp32 on CPU, {sub} of {s['batch']} batches "
            f"x {reps} reps ({el:.1f} s)"}


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--precision", choices=["tf32", "3xtf32"], default="tf32")
    ap.add_argument("--no-shapes", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--shapes", default="", help="comma list restricting the per-shape table")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the per-GPU batch (profiling runs on a small case)")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world, rank, local = dist_setup(args.gpus)
    dev = torch.cuda.current_device()
    torch.backends.cuda.matmul.allow_tf32 = True
    peaks = load_peaks()
    W = _pkg("workloads").WORKLOADS
    w = W[HEADLINE]
    if args.batch:
        import dataclasses

        shapes = dict(w.shapes, batch=args.batch)
        flops, nbytes = _pkg("workloads").cost_for(HEADLINE, **shapes)
        w = dataclasses.replace(w, shapes=shapes, flops=flops, min_bytes=nbytes)
    s = w.shapes

    if args.impl == "ours":
        ops = _pkg("ops")
        ops.set_precision(args.precision)
        op = ops.OPERATORS[w.pid].forward
        launches_per_step = 1
    else:
        op = None

    A, B = device_inputs(w, seed_offset=rank, **s)
    if args.impl == "ours":
        fn = lambda: op(A, B)
        impl_note = None
    else:
        try:
            fn, impl_note = reference_callable(HEADLINE, A, B)
        except Exception as e:  # reference module missing
            if rank == 0:
                print(json.dumps({"impl": "reference", "metric": METRIC,
                                  "unavailable": f"reference kernel not built: {e}"}))
            return

    clocks = ClockSampler(dev)
    clocks.start()
    total_ms, launch_ms = time_loop(fn, args.steps, args.warmup, world)
    # Keep sampling for a moment if the timed region was too short for nvidia-smi.
    if total_ms < 1500:
        t_end = time.perf_counter() + 1.0
        while time.perf_counter() < t_end:
            for _ in range(20):
                fn()
            torch.cuda.synchronize()
    clk = clocks.stop()
    ms_per_step = total_ms / args.steps
    value = world * w.flops / (ms_per_step / 1e3) / 1e12
    launch_ms = max_over_ranks(launch_ms, world)
    rl = roofline(w, launch_ms, peaks)
    traffic = load_traffic().get(f"{HEADLINE}:{args.precision}")
    rl["traffic"] = traffic
    rl["peak_source"] = peaks["source"]
    rl["peak_note"] = peaks["tf32_note"] if rl["bound"] == "tensor" else "MEASURED_PEAKS.json hbm_gbs"

    cublas = None
    if args.impl == "ours" and world == 1:
        cb = cublas_fn(HEADLINE, A, B)
        _, cb_ms = time_loop(cb, min(args.steps, 100), args.warmup)
        cublas = {"ms": round(cb_ms, 4), "tflops": round(w.flops / (cb_ms / 1e3) / 1e12, 2),
                  "what": "torch.matmul (cuBLAS) with TF32 allowed, same inputs, same GPU"}

    # ---- end to end through the public API, host buffers in the timed region
    e2e = None if args.no_e2e else end_to_end(args, w, A, B, op, world)

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "tf32" if args.precision == "tf32" else "3xtf32 (fp32-grade)",
        "data": "synthetic: N(0,1) fp32 from a per-rank seeded generator (no dataset)",
        "config": {"workload": "batched (BASELINE configs[2]; reference PID 3)"
                   + (f", batch overridden to {s['batch']}" if args.batch else ""),
                   "batch_per_gpu": s["batch"], "m": s["m"], "k": s["k"], "n": s["n"],
                   "global_batch": s["batch"] * world, "precision": args.precision,
                   "parallelism": f"batch-sharded x{world}, no communication",
                   "l2": f"inputs larger than L2 ({w.min_bytes / 1e9:.2f} GB touched per step)"},
        "roofline": rl, "e2e": e2e, "clocks": clk,
    }
    if cublas:
        line["cublas_tf32"] = cublas
    if args.impl == "ours":
        line["gpu_launches"] = launches_per_step * args.steps
    else:
        line["impl"] = "reference"
        line["reference"] = ("kernels/3_Batched_matrix_multiplication_best_kernel.cu:113 "
                             "batched_matmul_cuda, compiled unmodified for sm_100a")
    if args.impl == "ours" and not args.no_shapes:
        line["large_k_split"] = large_k_split(W, peaks, world, rank, min(args.steps, 100),
                                              args.warmup)
    if rank == 0 and world == 1 and args.impl == "ours" and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(w)
    if rank == 0 and world == 1 and args.impl == "ours" and not args.no_shapes:
        del A, B
        torch.cuda.empty_cache()
        only = set(x for x in args.shapes.split(",") if x)
        line["shapes"] = shape_table(W, peaks, only, ops)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def end_to_end(args, w, A, B, op, world):
    """The metric through the public API with pinned host inputs copied in and
    the result copied out inside the timed region."""
    s = w.shapes
    A_h = A.cpu().pin_memory()
    B_h = B.cpu().pin_memory()
    C_h = torch.empty(s["batch"], s["m"], s["n"], dtype=torch.float32).pin_memory()
    A_d = torch.empty_like(A)
    B_d = torch.empty_like(B)
    if args.impl == "ours":
        # The package's host-buffer entry: batch chunks streamed through
        # three CUDA streams (upload / GEMM / download overlap).
        ops = _pkg("ops")

        def e2e_step():
            ops.batched_matmul_from_host(A_h, B_h, out=C_h, chunks=8, synchronize=False)
    else:
        # The reference's entry point takes device tensors: copy in, call, copy out.
        e2e_call, _ = reference_callable(HEADLINE, A_d, B_d)

        def e2e_step():
            A_d.copy_(A_h, non_blocking=True)
            B_d.copy_(B_h, non_blocking=True)
            C = e2e_call()
            C_h.copy_(C, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 20))
    e2e_ms, _ = time_loop(e2e_step, e2e_steps, 2, world, per_launch=False)
    e2e_per = e2e_ms / e2e_steps
    e2e = {"value": round(world * w.flops / (e2e_per / 1e3) / 1e12, 3), "unit": "TFLOP/s",
           "ms_per_step": round(e2e_per, 3),
           "path": ("ops.batched_matmul_from_host: pinned host A, B -> C, 8 batch chunks "
                    "pipelined over upload / GEMM / download streams") if args.impl == "ours"
                   else "reference batched_matmul_cuda on device copies of pinned host A, B",
           "h2d_bytes_per_step": A.numel() * 4 + B.numel() * 4,
           "d2h_bytes_per_step": s["batch"] * s["m"] * s["n"] * 4}
    return e2e



def large_k_split(W, peaks, world, rank, steps, warmup):
    """Large-K config with K split across the ranks (strong scaling: total K
    fixed) and the 256x256 partials summed by one NCCL reduce to rank 0."""
    part = _pkg("partition").Partitioner.from_env()
    w = W["large_k"]
    m, n, k = w.shapes["m"], w.shapes["n"], w.shapes["k"]
    k0, k1 = part.k_range(k)
    g = torch.Generator(device="cuda").manual_seed(7000 + rank)
    A = torch.randn(m, k1 - k0, generator=g, device="cuda")
    B = torch.randn(k1 - k0, n, generator=g, device="cuda")
    fn = lambda: part.split_k_matmul(A, B, root=0)
    total, _ = time_loop(fn, steps, warmup, world, per_launch=False)
    ms = total / steps
    return {"workload": "large_k (BASELINE configs[3]; reference PID 6)", "k_total": k,
            "k_per_rank": k1 - k0, "ms": round(ms, 4),
            "gbs": round(w.min_bytes / (ms / 1e3) / 1e9, 1),
            "tflops": round(w.flops / (ms / 1e3) / 1e12, 2),
            "frac_hbm_1gpu": round(w.min_bytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 3),
            "collective": "local split-K GEMM, then NCCL reduce of the 256 KB partial to rank 0"
                          if world > 1 else "none (one GPU)",
            "scaling": "strong"}


def shape_table(W, peaks, only, ops):
    out = {}
    for name, w in W.items():
        if name == HEADLINE or (only and name not in only):
            continue
        args = device_inputs(w)
        op = ops.OPERATORS[w.pid].forward
        row = {"pid": w.pid, "shapes": w.shapes}
        ours = lambda: op(*args)
        # Let SM clocks recover from the previous (possibly power-capped) shape.
        torch.cuda.synchronize()
        time.sleep(0.5)
        k = adaptive_steps(ours)
        _, ms = time_loop(ours, k, 3)
        row["ours"] = roofline(w, ms, peaks)
        row["ours"]["ms"] = round(ms, 4)
        if w.useful_flops:
            row["ours"]["dense_equivalent_tflops"] = round(w.flops / (ms / 1e3) / 1e12, 2)
        if name in ("square", "transposed_b", "symmetric"):
            with ops.precision("3xtf32"):
                _, ms3 = time_loop(ours, k, 3)
            row["ours_3xtf32"] = {"ms": round(ms3, 4),
                                  "tflops": round(w.flops / (ms3 / 1e3) / 1e12, 2)}
        cb = cublas_fn(name, *args)
        _, msb = time_loop(cb, k, 3)
        fl = w.useful_flops or w.flops
        row["cublas_tf32"] = {"ms": round(msb, 4), "tflops": round(fl / (msb / 1e3) / 1e12, 2)}
        try:
            rf, note = reference_callable(name, *args)
            kr = adaptive_steps(rf, target_s=0.2, hi=200)
            _, msr = time_loop(rf, kr, 3)
            row["reference"] = {"ms": round(msr, 4),
                                "tflops": round(fl / (msr / 1e3) / 1e12, 2)}
            if note:
                row["reference"]["note"] = note
            row["speedup_vs_reference"] = round(msr / ms, 2)
        except Exception as e:
            row["reference"] = {"unavailable": str(e)[:120]}
        out[name] = row
        del args
        torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
