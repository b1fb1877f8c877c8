"""Run one benchmark workload a few times, for a profiler to capture.

    python cupilot-kernels_b200/profile_case.py --workload small_k --set m=8192 --set n=8192 \
        [--iters 3] [--precision tf32]

Inputs are generated on the device (seeded); each iteration is one operator
call, followed by a device synchronisation.  Shapes default to the
workload's benchmark config; --set overrides single dimensions (keep an
ncu capture small: a few GB on the device at most).
"""
from __future__ import annotations

import argparse
import importlib
import sys
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", required=True)
    ap.add_argument("--set", action="append", default=[], help="dim=value override")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--precision", default="tf32")
    args = ap.parse_args()
    W = importlib.import_module("cupilot-kernels_b200.workloads").WORKLOADS
    ops = importlib.import_module("cupilot-kernels_b200.ops")
    bench = importlib.import_module("bench")
    w = W[args.workload]
    over = {k: int(v) for k, v in (x.split("=") for x in args.set)}
    ops.set_precision(args.precision)
    call_args = bench.device_inputs(w, **over)
    op = ops.OPERATORS[w.pid].forward
    for _ in range(args.iters):
        op(*call_args)
        torch.cuda.synchronize()
    print(f"{args.workload} {dict(w.shapes, **over)} x{args.iters} ok")


if __name__ == "__main__":
    main()
