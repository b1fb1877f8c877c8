"""The benchmark configurations of the GEMM family, with seeded inputs.

Each workload names one operator (reference problem ID), its shapes, the
algorithmic work per call (2*M*N*K flops times batch; minimum fp32 bytes
with each operand read once and the output written once) and the bound
that work implies on B200.  Inputs are i.i.d. N(0, 1) fp32 drawn from a
CPU `torch.Generator` seeded per workload, so host copies and device copies
are bit-identical; structured operands follow the configs' recipes
(opposite triangle zeroed; symmetric = (X + X^T) / 2).

The shapes are the ones the benchmark configs state; the reference's own
problem definitions are not available, so these stand in for them.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, Tuple

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    pid: int
    shapes: Dict[str, int]
    seed: int
    make: Callable[..., Tuple[torch.Tensor, torch.Tensor]] = field(repr=False)
    flops: float
    min_bytes: float
    bound: str                 # "tensor" | "hbm"
    useful_flops: float = 0.0  # triangular ops: flops of the non-zero band

    def inputs(self, device="cpu", **override):
        """The operator's arguments (A, B — or input, weight, bias for the
        pointwise convolution), seeded on the CPU."""
        shapes = dict(self.shapes)
        shapes.update(override)
        g = torch.Generator().manual_seed(self.seed)
        args = self.make(g, **shapes)
        if device != "cpu":
            args = tuple(t.to(device) if isinstance(t, torch.Tensor) else t for t in args)
        return args


def _randn(g, *shape):
    return torch.randn(*shape, generator=g, dtype=torch.float32)


def _mk_nn(g, m, n, k):
    return _randn(g, m, k), _randn(g, k, n)


def _mk_tn(g, m, n, k):      # A stored (K, M)
    return _randn(g, k, m), _randn(g, k, n)


def _mk_nt(g, m, n, k):      # B stored (N, K)
    return _randn(g, m, k), _randn(g, n, k)


def _mk_tt(g, m, n, k):
    return _randn(g, k, m), _randn(g, n, k)


def _mk_bmm(g, batch, m, n, k):
    return _randn(g, batch, m, k), _randn(g, batch, k, n)


def _mk_3d(g, batch, m, n, k):
    return _randn(g, batch, m, k), _randn(g, k, n)


def _mk_4d(g, b, i, j, l, k):
    return _randn(g, b, i, j, l), _randn(g, l, k)


def _mk_diag(g, n):
    return _randn(g, n), _randn(g, n, n)


def _mk_upper(g, n):
    return torch.triu(_randn(g, n, n)), torch.triu(_randn(g, n, n))


def _mk_lower(g, n):
    return torch.tril(_randn(g, n, n)), torch.tril(_randn(g, n, n))


def _mk_sym(g, n):
    X = _randn(g, n, n)
    Y = _randn(g, n, n)
    return (X + X.T) / 2, (Y + Y.T) / 2


def _mk_gemv(g, m, k):
    return _randn(g, m, k), _randn(g, k, 1)


def _mk_scalar(g, m, n):
    return _randn(g, m, n), 2.5


def _mk_conv(g, batch, cin, cout, h, w):
    return _randn(g, batch, cin, h, w), _randn(g, cout, cin, 1, 1), _randn(g, cout)


def _conv_cost(batch, cin, cout, h, w):
    s = h * w
    flops = 2.0 * batch * cout * cin * s
    return flops, 4.0 * (batch * cin * s + cout * cin + cout + batch * cout * s)


def _gemm_cost(m, n, k, batch=1, a_shared=False, b_shared=False):
    flops = 2.0 * m * n * k * batch
    a = m * k * (1 if a_shared else batch)
    b = k * n * (1 if b_shared else batch)
    c = m * n * batch
    return flops, 4.0 * (a + b + c)


def _tri_useful(n):
    return 2.0 * n * (n + 1) * (n + 2) / 6.0


def _tri_cost(n):
    """Dense-equivalent flops, and the minimum bytes of a triangular product:
    the two operand triangles read once and the whole n x n output written
    (its masked triangle as zeros): 4 (n (n + 1) + n^2) bytes."""
    return 2.0 * n * n * n, 4.0 * (n * (n + 1) + n * n)


def _w(name, pid, shapes, seed, make, cost, bound, useful=0.0):
    flops, nbytes = cost
    return Workload(name, pid, shapes, seed, make, flops, nbytes, bound, useful)


WORKLOADS: Dict[str, Workload] = {}


def _add(w: Workload):
    WORKLOADS[w.name] = w


# square
_add(_w("square", 1, dict(m=2048, n=2048, k=2048), 0, _mk_nn, _gemm_cost(2048, 2048, 2048), "tensor"))
# Reference PID 2 (no benchmark config): its kernel hard-codes M = 2048,
# K = 8192, N = 4096 (kernels/2_Standard_matrix_multiplication_best_kernel.cu:16-18).
_add(_w("standard", 2, dict(m=2048, n=4096, k=8192), 19, _mk_nn, _gemm_cost(2048, 4096, 8192),
        "tensor"))
# transposed operands, M=1024, K=4096, N=2048
_add(_w("transposed_a", 16, dict(m=1024, n=2048, k=4096), 1, _mk_tn, _gemm_cost(1024, 2048, 4096), "tensor"))
_add(_w("transposed_b", 17, dict(m=1024, n=2048, k=4096), 2, _mk_nt, _gemm_cost(1024, 2048, 4096), "tensor"))
_add(_w("transposed_both", 18, dict(m=1024, n=2048, k=4096), 3, _mk_tt, _gemm_cost(1024, 2048, 4096), "tensor"))
# batched and 3-D
_add(_w("batched", 3, dict(batch=128, m=512, n=2048, k=1024), 4, _mk_bmm,
        _gemm_cost(512, 2048, 1024, 128), "tensor"))
_add(_w("tensor3d", 10, dict(batch=16, m=1024, n=768, k=2048), 5, _mk_3d,
        _gemm_cost(16 * 1024, 768, 2048), "tensor"))
# skewed shapes
_add(_w("small_k", 7, dict(m=16384, n=16384, k=32), 6, _mk_nn, _gemm_cost(16384, 16384, 32), "hbm"))
_add(_w("large_k", 6, dict(m=256, n=256, k=262144), 7, _mk_nn, _gemm_cost(256, 256, 262144), "hbm"))
_add(_w("tall_skinny", 9, dict(m=16384, n=16384, k=64), 8, _mk_nn, _gemm_cost(16384, 16384, 64), "hbm"))
_add(_w("irregular", 8, dict(m=8205, n=5921, k=2949), 9, _mk_nn, _gemm_cost(8205, 5921, 2949), "tensor"))
# structured operands at N=4096, and the 4-D product
_add(Workload("diag", 12, dict(n=4096), 10, _mk_diag, 4096.0 * 4096,
              4.0 * (4096 + 2 * 4096 * 4096), "hbm"))
_add(_w("upper_tri", 14, dict(n=4096), 11, _mk_upper, _tri_cost(4096), "tensor",
        _tri_useful(4096)))
_add(_w("lower_tri", 15, dict(n=4096), 12, _mk_lower, _tri_cost(4096), "tensor",
        _tri_useful(4096)))
_add(_w("symmetric", 13, dict(n=4096), 13, _mk_sym, _gemm_cost(4096, 4096, 4096), "tensor"))
_add(_w("tensor4d", 11, dict(b=16, i=256, j=512, l=256, k=768), 14, _mk_4d,
        _gemm_cost(16 * 256 * 512, 768, 256), "hbm"))


# Next rows (reference PIDs 4-5; no benchmark config names their sizes, so
# these are chosen HBM-bound sizes: a 1 GiB fp32 matrix streamed once).
_add(Workload("gemv", 4, dict(m=16384, k=16384), 15, _mk_gemv, 2.0 * 16384 * 16384,
              4.0 * (16384 * 16384 + 16384 + 16384), "hbm"))
_add(Workload("matrix_scalar", 5, dict(m=16384, n=16384), 16, _mk_scalar, 16384.0 * 16384,
              4.0 * 2 * 16384 * 16384, "hbm"))


# Next row (reference PID 87): the pointwise convolution.  No benchmark
# config names its size; out_channels = 128 is the size its kernel is tuned
# for (kernels/87_conv_pointwise_2D_best_kernel.cu:183), the rest is chosen:
# 16 images of 64 x 256 x 256, 0.27 GB in and 0.54 GB out (HBM-bound).
_add(_w("pointwise_conv", 87, dict(batch=16, cin=64, cout=128, h=256, w=256), 17, _mk_conv,
        _conv_cost(16, 64, 128, 256, 256), "hbm"))


# Next row (reference PID 97): attention, fp16.  The reference kernel only
# runs at seq 512 and dim 1024 (kernels/97_ScaledDotProductAttention_best_kernel.cu:9-10);
# batch and heads are chosen: 8 x 16 heads, 128 MB per tensor.
def _mk_sdpa(g, batch, heads, seq, dim):
    return tuple(_randn(g, batch, heads, seq, dim).half() for _ in range(3))


def _sdpa_cost(batch, heads, seq, dim):
    return 4.0 * batch * heads * seq * seq * dim, 2.0 * 4 * batch * heads * seq * dim


_add(_w("sdpa", 97, dict(batch=8, heads=16, seq=512, dim=1024), 18, _mk_sdpa,
        _sdpa_cost(8, 16, 512, 1024), "tensor"))


def cost_for(name: str, **shapes) -> Tuple[float, float]:
    """(flops, min_bytes) of a workload at overridden shapes."""
    w = WORKLOADS[name]
    s = dict(w.shapes)
    s.update(shapes)
    if name in ("square", "standard", "transposed_a", "transposed_b", "transposed_both",
                "small_k", "large_k", "tall_skinny", "irregular"):
        return _gemm_cost(s["m"], s["n"], s["k"])
    if name == "batched":
        return _gemm_cost(s["m"], s["n"], s["k"], s["batch"])
    if name == "tensor3d":
        return _gemm_cost(s["batch"] * s["m"], s["n"], s["k"])
    if name == "tensor4d":
        return _gemm_cost(s["b"] * s["i"] * s["j"], s["k"], s["l"])
    if name == "diag":
        n = s["n"]
        return float(n * n), 4.0 * (n + 2 * n * n)
    if name == "gemv":
        return 2.0 * s["m"] * s["k"], 4.0 * (s["m"] * s["k"] + s["m"] + s["k"])
    if name == "matrix_scalar":
        return float(s["m"] * s["n"]), 8.0 * s["m"] * s["n"]
    if name == "pointwise_conv":
        return _conv_cost(s["batch"], s["cin"], s["cout"], s["h"], s["w"])
    if name == "sdpa":
        return _sdpa_cost(s["batch"], s["heads"], s["seq"], s["dim"])
    n = s["n"]
    if name in ("upper_tri", "lower_tri"):
        return _tri_cost(n)
    return _gemm_cost(n, n, n)


def device_inputs(w: Workload, seed_offset: int = 0, device="cuda", **override):
    """Seeded N(0,1) inputs of a workload drawn directly on the device.

    Large configs (GBs of operands) are generated where they are used; the
    values differ from `Workload.inputs` (a CPU generator) but follow the
    same recipe per config (opposite triangle zeroed, symmetric =
    (X + X^T) / 2, attention in fp16).
    """
    g = torch.Generator(device=device).manual_seed(w.seed * 1000 + seed_offset)
    s = dict(w.shapes)
    s.update(override)
    r = lambda *sh: torch.randn(*sh, generator=g, device=device, dtype=torch.float32)
    n = w.name
    if n in ("square", "standard", "small_k", "large_k", "tall_skinny", "irregular"):
        return r(s["m"], s["k"]), r(s["k"], s["n"])
    if n == "transposed_a":
        return r(s["k"], s["m"]), r(s["k"], s["n"])
    if n == "transposed_b":
        return r(s["m"], s["k"]), r(s["n"], s["k"])
    if n == "transposed_both":
        return r(s["k"], s["m"]), r(s["n"], s["k"])
    if n == "batched":
        return r(s["batch"], s["m"], s["k"]), r(s["batch"], s["k"], s["n"])
    if n == "tensor3d":
        return r(s["batch"], s["m"], s["k"]), r(s["k"], s["n"])
    if n == "tensor4d":
        return r(s["b"], s["i"], s["j"], s["l"]), r(s["l"], s["k"])
    if n == "diag":
        return r(s["n"]), r(s["n"], s["n"])
    if n == "gemv":
        return r(s["m"], s["k"]), r(s["k"], 1)
    if n == "matrix_scalar":
        return r(s["m"], s["n"]), 2.5
    if n == "upper_tri":
        return torch.triu(r(s["n"], s["n"])), torch.triu(r(s["n"], s["n"]))
    if n == "lower_tri":
        return torch.tril(r(s["n"], s["n"])), torch.tril(r(s["n"], s["n"]))
    if n == "symmetric":
        X, Y = r(s["n"], s["n"]), r(s["n"], s["n"])
        return (X + X.T) / 2, (Y + Y.T) / 2
    if n == "pointwise_conv":
        return (r(s["batch"], s["cin"], s["h"], s["w"]), r(s["cout"], s["cin"], 1, 1),
                r(s["cout"]))
    if n == "sdpa":
        shape = (s["batch"], s["heads"], s["seq"], s["dim"])
        return tuple(r(*shape).half() for _ in range(3))
    raise KeyError(n)
