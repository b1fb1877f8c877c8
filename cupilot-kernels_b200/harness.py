"""Module-style boundary: each operator as a `torch.nn.Module`.

The reference's kernels were driven by a harness (absent from the
reference) that wrapped each Part-3 function in a module whose `forward`
called the compiled extension, next to a plain-PyTorch module computing the
same operator.  This file provides both sides for every operator here:

    from cupilot_kernels_b200 import harness        # (package dir: cupilot-kernels_b200)
    new = harness.model_new(3)                       # forward(A, B) -> ops.p3.forward(A, B)
    ref = harness.model_ref(3)                       # forward(A, B) -> torch.bmm(A, B)
    ok, err = harness.check(3, *harness.inputs(3, small=True))

`model_ref` is the operator's definition in plain torch (fp32; fp16 for
attention), written from the operator semantics stated with each reference
Part-3 function (file:line in `ops.OPERATORS`); `inputs` draws seeded inputs
from the benchmark workloads (`workloads.py`), optionally shrunk.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Tuple

import torch

from . import workloads


def _formula(pid: int) -> Callable:
    """The operator in plain torch, for comparison (not on the product path)."""
    tri_u = lambda A, B: torch.triu(torch.triu(A) @ torch.triu(B))       # kernels/14_...:135
    tri_l = lambda A, B: torch.tril(torch.tril(A) @ torch.tril(B))       # kernels/15_...:155
    table: Dict[int, Callable] = {
        1: torch.matmul, 2: torch.matmul, 6: torch.matmul, 7: torch.matmul, 8: torch.matmul,
        9: torch.matmul, 13: torch.matmul,
        3: torch.bmm,                                                     # kernels/3_...:113
        10: lambda A, B: torch.matmul(A, B),                              # kernels/10_...:180
        11: lambda A, B: torch.einsum("bijl,lk->bijk", A, B),             # kernels/11_...:132
        12: lambda a, B: a[:, None] * B,                                  # kernels/12_...:43
        14: tri_u, 15: tri_l,
        16: lambda A, B: A.t() @ B,                                       # kernels/16_...:124
        17: lambda A, B: A @ B.t(),                                       # kernels/17_...:267
        18: lambda A, B: A.t() @ B.t(),                                   # kernels/18_...:152
        4: torch.matmul,                                                  # kernels/4_...:84
        5: lambda A, s: A * s,                                            # kernels/5_...:47
        87: lambda x, w, b=None: torch.nn.functional.conv2d(             # kernels/87_...:451
            x, w.reshape(w.shape[0], -1, 1, 1), b),
        97: lambda q, k, v: torch.softmax(                                # kernels/97_...:256
            (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1]), -1
        ) @ v.float(),
    }
    return table[pid]


class ModelNew(torch.nn.Module):
    """forward(*inputs) runs the B200 operator for one reference problem ID."""

    def __init__(self, pid: int):
        super().__init__()
        from . import ops

        self.pid = pid
        self.op = ops.OPERATORS[pid]

    def forward(self, *args):
        return self.op.forward(*args)


class ModelRef(torch.nn.Module):
    """forward(*inputs) computes the same operator in plain torch."""

    def __init__(self, pid: int):
        super().__init__()
        self.pid = pid
        self.fn = _formula(pid)

    def forward(self, *args):
        return self.fn(*args)


def model_new(pid: int) -> ModelNew:
    return ModelNew(pid)


def model_ref(pid: int) -> ModelRef:
    return ModelRef(pid)


def pids():
    """Problem IDs with both a module and a benchmark workload."""
    have = {w.pid for w in workloads.WORKLOADS.values()}
    return sorted(p for p in have if p in (1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17,
                                            18, 87, 97))


# Shrunk shapes for quick checks (same structure as the workload's config).
_SMALL = {
    "square": dict(m=256, n=256, k=256), "standard": dict(m=256, n=384, k=512), "batched": dict(batch=4, m=128, n=256, k=128),
    "small_k": dict(m=512, n=384, k=32), "large_k": dict(m=64, n=64, k=8192),
    "tall_skinny": dict(m=512, n=512, k=64), "irregular": dict(m=205, n=121, k=149),
    "tensor3d": dict(batch=2, m=128, n=96, k=256), "tensor4d": dict(b=2, i=4, j=8, l=64, k=96),
    "diag": dict(n=300), "upper_tri": dict(n=300), "lower_tri": dict(n=300), "symmetric": dict(n=300),
    "transposed_a": dict(m=128, n=256, k=512), "transposed_b": dict(m=128, n=256, k=512),
    "transposed_both": dict(m=128, n=256, k=512), "gemv": dict(m=1000, k=777),
    "matrix_scalar": dict(m=100, n=300), "pointwise_conv": dict(batch=2, cin=24, cout=40, h=9, w=11),
    "sdpa": dict(batch=1, heads=2, seq=200, dim=128),
}


def inputs(pid: int, small: bool = False, device: str = "cuda") -> Tuple:
    """Seeded inputs of the benchmark workload for `pid` (shrunk if `small`)."""
    w = next(w for w in workloads.WORKLOADS.values() if w.pid == pid)
    over = _SMALL.get(w.name, {}) if small else {}
    return w.inputs(device=device, **over)


def check(pid: int, *args, tol: float | None = None) -> Tuple[bool, float]:
    """ModelNew against ModelRef on the same inputs: (passed, relative Frobenius error).

    Tolerances: 1e-2 (TF32 operators), exact for the fp32 element-wise
    operators (PIDs 5, 12), 5e-3 for fp16 attention.
    """
    out = model_new(pid)(*args).double()
    ref = model_ref(pid)(*[a.double() if torch.is_tensor(a) and a.dtype == torch.float32 else a
                            for a in args]).double()
    if pid in (5, 12):
        ref = model_ref(pid)(*args).double()   # one fp32 rounding, compared bit for bit
    num = torch.linalg.vector_norm(out - ref).item()
    den = torch.linalg.vector_norm(ref).item()
    err = num / den if den else num
    if tol is None:
        tol = 0.0 if pid in (5, 12) else (5e-3 if pid == 97 else 1e-2)
    return err <= tol, err
