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
`parity` is the relative Frobenius error of a sampled subset of the measured
output against a float64 product on the GPU.  Extra keys:
  large_k_split  the large-K config with K split across the ranks and the
                 partials summed on rank 0 by the peer-memory reduction;
                 at N > 1 its one-GPU time and efficiency t1 / (N tN)
  sharded        the 3-D and 4-D configs with the batch split across ranks
  shapes         (N = 1) every other config, compact: [ours ms, achieved,
                 TF|GB, fraction of roofline, cuBLAS ms, parity]
Inputs smaller than 3x L2 rotate over several seeded sets, so every call
reads its operands from HBM.

--impl reference runs the reference's own CUDA kernel for the workload
(kernels/3_Batched_matrix_multiplication_best_kernel.cu:113, compiled
unmodified for sm_100a into oracle/_ref) through its own entry point, on
every rank, timed the same way; at N = 1 its `shapes` holds the reference
kernel of every other config on the same inputs ([ms, parity]).
"""
from __future__ import annotations

import argparse
import importlib
import itertools
import json
import math
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
L2_BYTES = 126e6   # B200 L2


def input_sets(nbytes, cap=8):
    """How many distinct input sets to rotate through so that each call's
    inputs have left L2 since their last use (at least 3x L2 touched per
    rotation); 1 when one set is already larger than that."""
    if nbytes >= 3 * L2_BYTES:
        return 1
    return int(min(cap, math.ceil(3 * L2_BYTES / max(nbytes, 1.0))))


def rotating(call, sets):
    """A no-argument step that calls `call(*set)` cycling over `sets`."""
    it = itertools.cycle(sets)
    return lambda: call(*next(it))


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


def workload_sets(w, nsets=None, **shapes):
    """`nsets` seeded input sets of a workload (enough to defeat L2 if None)."""
    if nsets is None:
        nsets = input_sets(_pkg("workloads").cost_for(w.name, **shapes)[1] if shapes
                           else w.min_bytes)
    return [device_inputs(w, i, **shapes) for i in range(nsets)]


# ---------------------------------------------------------------- parity (sampled, fp64 on the GPU)
def _rows(m, count=48):
    idx = torch.linspace(0, m - 1, steps=min(count, m)).round().long().tolist()
    return sorted(set(idx + list(range(max(0, m - 8), m))))


def _rel(got, ref):
    got = got.double()
    den = float(ref.norm())
    num = float((got - ref).norm())
    return num / den if den else num


def sampled_parity(name, args, out):
    """Relative Frobenius error of a sampled subset of `out` (rows spread over
    M, the last rows included) against a float64 product on the GPU; 0.0
    means bit-identical for the one-rounding element-wise operators.  A check
    on the measured output, not part of the timed work."""
    d = torch.float64
    A = args[0]
    B = args[1] if len(args) > 1 else None
    if name in ("square", "standard", "small_k", "large_k", "tall_skinny", "irregular",
                "symmetric"):
        r = _rows(A.shape[0])
        return _rel(out[r], A[r].to(d) @ B.to(d))
    if name in ("transposed_a", "transposed_both"):
        r = _rows(A.shape[1])
        Bd = B.to(d) if name == "transposed_a" else B.to(d).T
        return _rel(out[r], A[:, r].to(d).T @ Bd)
    if name == "transposed_b":
        r = _rows(A.shape[0])
        return _rel(out[r], A[r].to(d) @ B.to(d).T)
    if name == "batched":
        sel = [0, A.shape[0] // 2, A.shape[0] - 1]
        return _rel(out[sel], torch.matmul(A[sel].to(d), B[sel].to(d)))
    if name in ("tensor3d", "tensor4d"):
        l = A.shape[-1]
        Af = A.reshape(-1, l)
        r = _rows(Af.shape[0], 256)
        return _rel(out.reshape(Af.shape[0], -1)[r], Af[r].to(d) @ B.to(d))
    if name in ("upper_tri", "lower_tri"):
        tri = torch.triu if name == "upper_tri" else torch.tril
        r = _rows(A.shape[0])
        ref = tri(A).to(d)[r] @ tri(B).to(d)
        cols = torch.arange(A.shape[0], device=A.device)[None, :]
        rows = torch.tensor(r, device=A.device)[:, None]
        keep = cols >= rows if name == "upper_tri" else cols <= rows
        ref = torch.where(keep, ref, torch.zeros_like(ref))
        masked = out[~torch.ones_like(out, dtype=torch.bool).triu() if name == "upper_tri"
                     else ~torch.ones_like(out, dtype=torch.bool).tril()]
        if torch.count_nonzero(masked).item():
            return float("inf")          # the masked triangle must be exactly zero
        return _rel(out[r], ref)
    if name == "diag":
        return 0.0 if torch.equal(out, A[:, None] * B) else _rel(out, (A[:, None] * B).to(d))
    if name == "matrix_scalar":
        return 0.0 if torch.equal(out, A * B) else _rel(out, (A * B).to(d))
    if name == "gemv":
        r = _rows(A.shape[0])
        return _rel(out[r], A[r].to(d) @ B.to(d))
    if name == "pointwise_conv":
        x, wt, bias = args
        n, c = x.shape[0], x.shape[1]
        ref = wt.reshape(wt.shape[0], c).to(d) @ x[n - 1].reshape(c, -1).to(d) + \
            bias.to(d)[:, None]
        return _rel(out[n - 1].reshape(ref.shape), ref)
    if name == "sdpa":
        q, k, v = (t[-1, -1].to(d) for t in args)
        p = torch.softmax(q @ k.T / math.sqrt(q.shape[-1]), dim=-1)
        return _rel(out[-1, -1], p @ v)
    raise KeyError(name)


def _sig(x, digits=3):
    """Round to `digits` significant figures (compact JSON)."""
    if x is None or x == 0 or not math.isfinite(x):
        return x
    return round(x, digits - 1 - int(math.floor(math.log10(abs(x)))))


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
    "gemv": 4, "matrix_scalar": 5, "standard": 2,
    "square": 1, "batched": 3, "large_k": 6, "small_k": 7, "irregular": 8, "tall_skinny": 9,
    "tensor3d": 10, "tensor4d": 11, "diag": 12, "symmetric": 13, "upper_tri": 14,
    "lower_tri": 15, "transposed_a": 16, "transposed_b": 17, "transposed_both": 18,
    "pointwise_conv": 87, "sdpa": 97,
}


def reference_callable(name, A, B, *rest):
    from oracle import build_ref

    if name == "gemv" and not (A.shape[1] >= 12288 and A.shape[1] % 4 == 0):
        # K4's main loop bound `num_vectors - blockDim.x*3` (kernels/4_...:22)
        # mixes int with unsigned: below 3072 float4s per row (K < 12288 at
        # its 1024 threads) it wraps to a huge value and the loop reads far
        # past the row.  It runs only where the bound cannot wrap.
        raise RuntimeError("K4 reads out of bounds for K < 12288 (kernels/4_...:22); not run")
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
    ap.add_argument("--no-extras", action="store_true",
                    help="skip large-K split and 3-D/4-D sharding legs")
    ap.add_argument("--shapes", default="", help="comma list restricting the per-shape table")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the per-GPU batch (profiling runs on a small case)")
    ap.add_argument("--profile-case", default="",
                    help="run only this workload (name) for --steps calls, untimed: the "
                         "command an ncu capture of one config wraps")
    ap.add_argument("--profile-impl", choices=["ours", "cublas", "fused"], default="ours",
                    help="--profile-case: our operator, the same math through cuBLAS, or (large_k) "
                         "the one-kernel cross-GPU K split with two ranks emulated on one GPU")
    ap.add_argument("--set", action="append", default=[],
                    help="dim=value override of the --profile-case workload's shape")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3 and not args.profile_case:
        args.warmup = 3

    world, rank, local = dist_setup(args.gpus)
    dev = torch.cuda.current_device()
    torch.backends.cuda.matmul.allow_tf32 = True
    peaks = load_peaks()
    W = _pkg("workloads").WORKLOADS
    if args.profile_case:
        return profile_case(W, args)
    w = W[HEADLINE]
    if args.batch:
        import dataclasses

        shapes = dict(w.shapes, batch=args.batch)
        flops, nbytes = _pkg("workloads").cost_for(HEADLINE, **shapes)
        w = dataclasses.replace(w, shapes=shapes, flops=flops, min_bytes=nbytes)
    s = w.shapes

    ops = None
    if args.impl == "ours":
        ops = _pkg("ops")
        ops.set_precision(args.precision)
        op = ops.OPERATORS[w.pid].forward
    else:
        op = None

    A, B = device_inputs(w, seed_offset=rank, **s)
    if args.impl == "ours":
        fn = lambda: op(A, B)
    else:
        try:
            fn, _ = reference_callable(HEADLINE, A, B)
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
    rl["traffic"] = load_traffic().get(f"{HEADLINE}:{args.precision}")
    rl["peak_source"] = peaks["source"]
    par = _sig(sampled_parity(HEADLINE, (A, B), fn()))

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "tf32" if args.precision == "tf32" else "3xtf32",
        "data": "synthetic N(0,1) fp32, seeded per rank",
        "config": {"workload": "batched (BASELINE configs[2], ref PID 3)"
                   + (f", batch {s['batch']}" if args.batch else ""),
                   "batch_per_gpu": s["batch"], "m": s["m"], "k": s["k"], "n": s["n"],
                   "global_batch": s["batch"] * world, "parallelism": f"batch x{world}, no comm",
                   "l2": f"inputs > L2 ({w.min_bytes / 1e9:.2f} GB/step)"},
        "roofline": rl, "parity": par, "clocks": clk,
    }
    if args.impl == "ours":
        line["gpu_launches"] = args.steps        # one engine launch per step
        line["e2e"] = None if args.no_e2e else end_to_end(args, w, A, B, op, world)
    else:
        line["impl"] = "reference"
        line["reference"] = "kernels/3_...:113 batched_matmul_cuda, unmodified, sm_100a"
        line["e2e"] = None if args.no_e2e else end_to_end(args, w, A, B, op, world)
    if args.impl == "ours" and world == 1:
        cb = cublas_fn(HEADLINE, A, B)
        _, cb_ms = time_loop(cb, min(args.steps, 100), args.warmup)
        line["cublas_tf32_ms"] = round(cb_ms, 4)
    del A, B, fn
    torch.cuda.empty_cache()
    if args.impl == "ours" and not args.no_extras:
        line["large_k_split"] = large_k_split(W, peaks, world, rank, args.warmup)
        line["sharded"] = sharded(W, peaks, world, rank, args.warmup)
    if rank == 0 and world == 1 and args.impl == "ours" and not args.no_cpu:
        w_head = W[HEADLINE]
        line["cpu_baseline"] = cpu_baseline(w_head)
    if rank == 0 and world == 1 and not args.no_shapes:
        only = set(x for x in args.shapes.split(",") if x)
        if args.impl == "ours":
            line["shapes"] = shape_table(W, peaks, only, ops)
        else:
            line["shapes"] = reference_shape_table(W, only)
    if rank == 0:
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def profile_case(W, args):
    """One workload called --warmup + --steps times, each call followed by a
    device synchronisation (no timing): the command the committed ncu
    summaries wrap.  --set dim=value shrinks a dimension for a small capture."""
    ops = _pkg("ops")
    ops.set_precision(args.precision)
    w = W[args.profile_case]
    over = {k: int(v) for k, v in (x.split("=") for x in args.set)}
    ins = device_inputs(w, **over)
    if args.profile_impl == "fused":
        # b2g_gemm_splitk_peer with two ranks emulated on this GPU, one after
        # the other (rank 1, then the root), the device synchronised between
        # them: no kernel waits for another that runs beside it.
        capi = _pkg("capi")
        nat = importlib.import_module(PKG).native()
        A, B = ins[0], ins[1]
        h = A.shape[1] // 2
        halves = [(A[:, :h].contiguous(), B[:h].contiguous()), (A[:, h:].contiguous(), B[h:].contiguous())]
        mb = [capi.peer_mailbox_create(A.shape[0] * B.shape[1], 2)[0] for _ in range(2)]
        for epoch in range(1, args.warmup + args.steps + 1):
            for rk in (1, 0):
                nat.splitk_peer_matmul(*halves[rk], mb, rk, 0, epoch)
                torch.cuda.synchronize()
        for ptr in mb:
            capi.peer_mailbox_destroy(ptr)
        print(json.dumps({"profile_case": w.name, "impl": "fused", "shapes": dict(w.shapes, **over),
                          "calls": 2 * (args.warmup + args.steps),
                          "device_error": ops.read_device_error(torch.cuda.current_device())}))
        return
    if args.profile_impl == "cublas":
        op = lambda *a: cublas_fn(w.name, *a)()
    else:
        op = ops.OPERATORS[w.pid].forward
    for _ in range(args.warmup + args.steps):
        op(*ins)
        torch.cuda.synchronize()
    print(json.dumps({"profile_case": w.name, "impl": args.profile_impl,
                      "shapes": dict(w.shapes, **over),
                      "calls": args.warmup + args.steps,
                      "device_error": ops.read_device_error(torch.cuda.current_device())}))


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
    return {"value": round(world * w.flops / (e2e_per / 1e3) / 1e12, 3), "unit": "TFLOP/s",
            "ms_per_step": round(e2e_per, 3),
            "path": "ops.batched_matmul_from_host, pinned host A,B->C, 8 chunks on 3 streams"
                    if args.impl == "ours" else "K3 on device copies of pinned host A,B",
            "h2d_bytes_per_step": A.numel() * 4 + B.numel() * 4,
            "d2h_bytes_per_step": s["batch"] * s["m"] * s["n"] * 4}


def _steps_for(ms_estimate, target_ms=300.0, lo=20, hi=400):
    return int(min(hi, max(lo, target_ms / max(ms_estimate, 1e-3))))


def large_k_split(W, peaks, world, rank, warmup):
    """Large-K config with K split across the ranks (strong scaling: total K
    fixed).  At N > 1 each step is one kernel per rank
    (b2g_gemm_splitk_peer): the rank's K-slice product, then, in the same
    kernel, its 256 x 256 partial pushed to rank 0 over peer memory and
    summed there.  Inputs rotate over enough sets that
    each call reads its operands from HBM.  At N > 1 rank 0 also times the
    whole config on its own GPU, for the efficiency t1 / (N t_N)."""
    part = _pkg("partition").Partitioner.from_env()
    w = W["large_k"]
    m, n, k = w.shapes["m"], w.shapes["n"], w.shapes["k"]
    k0, k1 = part.k_range(k)
    # Set 0: slices of one full A, B (the same on every rank) for the parity check.
    g = torch.Generator(device="cuda").manual_seed(7000)
    A_full = torch.randn(m, k, generator=g, device="cuda")
    B_full = torch.randn(k, n, generator=g, device="cuda")
    per_rank = 4.0 * (m + n) * (k1 - k0)
    nsets = input_sets(per_rank)
    sets = [(A_full[:, k0:k1].contiguous(), B_full[k0:k1].contiguous())]
    for i in range(1, nsets):
        gi = torch.Generator(device="cuda").manual_seed(7000 + 100 * i + rank)
        sets.append((torch.randn(m, k1 - k0, generator=gi, device="cuda"),
                     torch.randn(k1 - k0, n, generator=gi, device="cuda")))
    step = rotating(lambda A, B: part.split_k_matmul(A, B, root=0), sets)
    step()                                           # creates the mailboxes (collective)
    torch.cuda.synchronize()
    steps = 200
    total, _ = time_loop(step, steps, warmup, world, per_launch=False)
    ms_serial = total / steps
    # The same steps as two kernels (GEMM, then the stand-alone peer-memory
    # sum) on the same mailboxes, for comparison with the fused kernel.
    step2 = rotating(lambda A, B: part.split_k_matmul(A, B, root=0, method="peer"), sets)
    total2, _ = time_loop(step2, steps, warmup, world, per_launch=False)
    ms_two = total2 / steps
    # Pipelined: each step's cross-GPU sum runs on a side stream and overlaps
    # the next step's GEMM; the timed region ends after the last sum (join).
    astep = rotating(lambda A, B: part.split_k_matmul_async(A, B, root=0), sets)

    def pipelined():
        astep()

    for _ in range(warmup):
        pipelined()
    part.join()
    torch.cuda.synchronize()
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        pipelined()
    part.join()
    ev1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms_pipe = max_over_ranks(ev0.elapsed_time(ev1), world) / steps
    ms = ms_serial
    C = part.split_k_matmul(*sets[0], root=0)
    torch.cuda.synchronize()
    out = {"ms": round(ms, 4), "tflops": round(w.flops / (ms / 1e3) / 1e12, 2),
           "gbs": round(w.min_bytes / (ms / 1e3) / 1e9, 1), "k_per_rank": k1 - k0,
           "input_sets": nsets,
           "reduce": "fused into the GEMM kernel: peer-memory push to rank 0, one step at a time"
                     if world > 1 else "none (one GPU)"}
    if world > 1:
        out["ms_two_kernels"] = round(ms_two, 4)  # GEMM + stand-alone peer sum (information)
        out["ms_pipelined"] = round(ms_pipe, 4)   # sums on a side stream (information)
    if rank == 0:
        out["parity"] = _sig(_rel(C, A_full.double() @ B_full.double()))
    if world > 1:
        t1 = None
        if rank == 0:
            ops = _pkg("ops")
            one = lambda: ops.p6.forward(A_full, B_full)
            tot1, _ = time_loop(one, 100, warmup)
            t1 = tot1 / 100
        barrier(world)
        if rank == 0:
            out["ms_1gpu"] = round(t1, 4)
            out["eff"] = round(t1 / (world * ms), 3)
    del sets, A_full, B_full
    torch.cuda.empty_cache()
    return out


def sharded(W, peaks, world, rank, warmup):
    """3-D (K10) and 4-D (K11) products with the batch sharded over the ranks
    (strong scaling: the config's total is fixed; rank r computes its
    contiguous batch slice with no communication).  At N > 1 rank 0 also
    times the whole config on its own GPU for the efficiency t1 / (N t_N)."""
    part = _pkg("partition").Partitioner.from_env()
    ops = _pkg("ops")
    out = {}
    for name, bkey in (("tensor3d", "batch"), ("tensor4d", "b")):
        w = W[name]
        total_b = w.shapes[bkey]
        b0, b1 = part.batch_range(total_b)
        shapes = dict(w.shapes)
        shapes[bkey] = b1 - b0
        op = ops.OPERATORS[w.pid].forward
        sets = workload_sets(w, **shapes)
        step = rotating(op, sets)
        steps = 50
        tot, _ = time_loop(step, steps, warmup, world, per_launch=False)
        ms = tot / steps
        row = {"ms": round(ms, 4), "tflops": round(w.flops / (ms / 1e3) / 1e12, 2),
               "batch_per_rank": b1 - b0}
        del sets, step
        torch.cuda.empty_cache()
        if world > 1:
            t1 = None
            if rank == 0:
                full = workload_sets(w)
                tot1, _ = time_loop(rotating(op, full), steps, warmup)
                t1 = tot1 / steps
                del full
                torch.cuda.empty_cache()
            barrier(world)
            if rank == 0:
                row["ms_1gpu"] = round(t1, 4)
                row["eff"] = round(t1 / (world * ms), 3)
        out[name] = row
    return out


SHAPE_COLS = ["ms", "achieved", "unit", "frac", "cublas_ms", "parity"]
X3_SHAPES = ("square", "transposed_b", "symmetric")


def shape_table(W, peaks, only, ops):
    """Every other workload on one GPU: [ours ms, achieved (TF: TFLOP/s or GB:
    GB/s), fraction of its roofline, cuBLAS ms, sampled parity].  Inputs
    rotate over enough sets that each call reads its operands from HBM; the
    cuBLAS column uses the same sets.  `<name>@3x` rows are 3xTF32 against
    cuBLAS fp32 (TF32 off).  The full rows also go to stderr."""
    out = {"cols": SHAPE_COLS}
    for name, w in W.items():
        if name == HEADLINE or (only and name not in only):
            continue
        sets = workload_sets(w)
        op = ops.OPERATORS[w.pid].forward
        ours = rotating(op, sets)
        torch.cuda.synchronize()
        time.sleep(0.5)          # let SM clocks recover from the previous power-capped shape
        k = adaptive_steps(ours)
        _, ms = time_loop(ours, k, 3)
        rl = roofline(w, ms, peaks)
        par = _sig(sampled_parity(name, sets[0], op(*sets[0])))
        cb = rotating(lambda *a: cublas_fn(name, *a)(), sets)
        _, msb = time_loop(cb, k, 3)
        unit = "TF" if rl["unit"] == "TFLOP/s" else "GB"
        out[name] = [_sig(ms, 4), _sig(rl["achieved"], 4), unit, _sig(rl["frac"]), _sig(msb, 4),
                     par]
        print(json.dumps({"shape": name, "ours": rl, "ours_ms": ms, "cublas_ms": msb,
                          "parity": par, "shapes": w.shapes}), file=sys.stderr)
        if name in X3_SHAPES:
            with ops.precision("3xtf32"):
                _, ms3 = time_loop(ours, k, 3)
                par3 = _sig(sampled_parity(name, sets[0], op(*sets[0])))
            torch.backends.cuda.matmul.allow_tf32 = False
            _, msf = time_loop(cb, k, 3)
            torch.backends.cuda.matmul.allow_tf32 = True
            tf3 = w.flops / (ms3 / 1e3) / 1e12
            out[name + "@3x"] = [_sig(ms3, 4), _sig(tf3, 4), "TF",
                                 _sig(tf3 / peaks["tf32_tflops"]), _sig(msf, 4), par3]
        del sets, ours, cb
        torch.cuda.empty_cache()
    return out


def reference_shape_table(W, only):
    """The reference's own kernel per workload (compiled unmodified), on the
    same rotating input sets: {name: [ms, parity]} (+ a note where it runs
    outside its contract)."""
    out = {"cols": ["ref_ms", "parity"]}
    for name, w in W.items():
        if name == HEADLINE or (only and name not in only):
            continue
        sets = workload_sets(w)
        try:
            calls = [reference_callable(name, *a) for a in sets]
        except Exception as e:
            out[name] = [None, str(e)[:80]]
            continue
        it = itertools.cycle(calls)
        rf = lambda: next(it)[0]()
        torch.cuda.synchronize()
        time.sleep(0.3)
        kr = adaptive_steps(rf, target_s=0.2, hi=200)
        _, msr = time_loop(rf, kr, 3)
        par = _sig(sampled_parity(name, sets[0], calls[0][0]()))
        out[name] = [_sig(msr, 4), par] + ([calls[0][1]] if calls[0][1] else [])
        del sets, calls, it
        torch.cuda.empty_cache()
    return out


if __name__ == "__main__":
    main()
