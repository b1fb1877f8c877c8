"""Parity at the benchmark configs' own sizes.

Every benchmark config runs at its full shape, in both precision modes, and
is checked two ways:

* the whole output against a float64 product computed on the GPU (torch's
  float64 matmul, an independent library path), row chunk by row chunk,
  as one relative Frobenius norm over all of C;
* a sampled subset against the CPU fp64 oracle (oracle/gemm_oracle.py):
  whole batches (the last included) for the batched config, rows spread
  over M (the last tile row included) for the skewed shapes, rows on both
  sides of the 2^31-byte output offset for the 4-D product, and the two
  corner blocks of the triangular products (which depend only on the
  matching corner blocks of A and B).

Triangular outputs must be exactly zero in the masked triangle over all of
C.  Tolerances: relative Frobenius 1e-2 (TF32) and 1e-3 (3xTF32).

The configs reach the code paths small shapes do not: the dynamic unit
schedule with thousands of units (its unit ring wraps many times), batched
units on the dynamic schedule, output offsets past 2^31 bytes, the
triangular unit table with split K pieces, and split-K over 74 pieces.
Reference sites: kernels/1_...:189, 2_...:16-18,117, 3_...:113, 6_...:128, 7_...:80,
8_...:155, 9_...:145, 10_...:180, 11_...:132,165, 13_...:134, 14_...:135,
15_...:155, 16_...:124, 17_...:267, 18_...:152.
"""
import numpy as np
import pytest
import torch

from conftest import import_pkg
from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = O.TOL
MODES = ["tf32", "3xtf32"]
CONFIGS = ["square", "standard", "transposed_a", "transposed_b", "transposed_both", "batched", "tensor3d",
           "small_k", "large_k", "tall_skinny", "irregular", "upper_tri", "lower_tri",
           "symmetric", "tensor4d"]


def _np(t):
    return t.detach().cpu().numpy()


def _chunks(n, rows):
    return [(r0, min(n, r0 + rows)) for r0 in range(0, n, rows)]


class Fro:
    """Relative Frobenius norm accumulated over chunks, in float64 on the GPU."""

    def __init__(self):
        self.num = 0.0
        self.den = 0.0

    def add(self, got, ref):
        d = got.double() - ref
        self.num += float((d * d).sum())
        self.den += float((ref * ref).sum())

    def value(self):
        return (self.num / self.den) ** 0.5 if self.den > 0 else self.num ** 0.5


def full_check(name, A, B, C):
    """Relative Frobenius norm of all of C against a float64 GPU product."""
    f = Fro()
    d = torch.float64
    if name in ("square", "standard", "small_k", "large_k", "tall_skinny", "irregular",
                "symmetric"):
        Bd = B.to(d)
        for r0, r1 in _chunks(A.shape[0], 2048):
            f.add(C[r0:r1], A[r0:r1].to(d) @ Bd)
    elif name == "transposed_a":
        Bd = B.to(d)
        for r0, r1 in _chunks(A.shape[1], 2048):
            f.add(C[r0:r1], A[:, r0:r1].to(d).T @ Bd)
    elif name == "transposed_b":
        Bt = B.to(d).T
        for r0, r1 in _chunks(A.shape[0], 2048):
            f.add(C[r0:r1], A[r0:r1].to(d) @ Bt)
    elif name == "transposed_both":
        Bt = B.to(d).T
        for r0, r1 in _chunks(A.shape[1], 2048):
            f.add(C[r0:r1], A[:, r0:r1].to(d).T @ Bt)
    elif name == "batched":
        for b in range(A.shape[0]):
            f.add(C[b], A[b].to(d) @ B[b].to(d))
    elif name in ("tensor3d", "tensor4d"):
        l = A.shape[-1]
        Af = A.reshape(-1, l)
        Cf = C.reshape(Af.shape[0], -1)
        Bd = B.to(d)
        for r0, r1 in _chunks(Af.shape[0], 65536):
            f.add(Cf[r0:r1], Af[r0:r1].to(d) @ Bd)
    elif name in ("upper_tri", "lower_tri"):
        up = name == "upper_tri"
        tri = torch.triu if up else torch.tril
        At, Bt = tri(A).to(d), tri(B).to(d)
        for r0, r1 in _chunks(A.shape[0], 1024):
            f.add(C[r0:r1], tri(At[r0:r1] @ Bt, diagonal=r0))
    else:
        raise KeyError(name)
    return f.value()


def sample_check(name, A, B, C):
    """Relative Frobenius norm of a sampled subset of C against the CPU oracle."""
    errs = []
    if name in ("square", "standard", "small_k", "large_k", "tall_skinny", "irregular",
                "symmetric", "transposed_b"):
        m = A.shape[0]
        rows = _sample_rows(m, 512)
        ref = O.BY_PID[_pid(name)](_np(A[rows]), _np(B))
        errs.append(O.rel_fro(_np(C[rows]), ref))
    elif name in ("transposed_a", "transposed_both"):
        m = A.shape[1]
        rows = _sample_rows(m, 256)
        ref = O.BY_PID[_pid(name)](_np(A[:, rows]), _np(B))
        errs.append(O.rel_fro(_np(C[rows]), ref))
    elif name == "batched":
        nb = A.shape[0]
        sel = sorted(set(np.linspace(0, nb - 1, 8).astype(int).tolist()))
        ref = O.batched(_np(A[sel]), _np(B[sel]))
        errs.append(O.rel_fro(_np(C[sel]), ref))
    elif name == "tensor3d":
        sel = [0, A.shape[0] - 1]                     # two whole batch entries
        ref = O.tensor3d(_np(A[sel]), _np(B))
        errs.append(O.rel_fro(_np(C[sel]), ref))
    elif name == "tensor4d":
        l, k = A.shape[-1], B.shape[1]
        Af = A.reshape(-1, l)
        Cf = C.reshape(Af.shape[0], k)
        rows_total = Af.shape[0]
        cut = (1 << 31) // (k * 4)                    # first row whose offset passes 2^31 bytes
        rows = sorted(set(list(range(cut - 256, cut + 256)) + list(range(rows_total - 256, rows_total))
                          + _sample_rows(rows_total, 256)))
        ref = O.tensor4d(_np(Af[rows]).reshape(1, 1, len(rows), l), _np(B))
        errs.append(O.rel_fro(_np(Cf[rows]), ref.reshape(len(rows), k)))
    elif name in ("upper_tri", "lower_tri"):
        n = A.shape[0]
        s = 1024
        f = O.upper_tri if name == "upper_tri" else O.lower_tri
        # C's corner blocks depend only on the matching corner blocks of A and B
        # (the K range of entry (i, j) lies between i and j).
        for sl in (slice(0, s), slice(n - s, n)):
            errs.append(O.rel_fro(_np(C[sl, sl]), f(_np(A[sl, sl]), _np(B[sl, sl]))))
    else:
        raise KeyError(name)
    return max(errs)


def _pid(name):
    return import_pkg("workloads").WORKLOADS[name].pid


def _sample_rows(m, count):
    """`count` rows spread over [0, m), the last 128 (the last tile row) included."""
    g = np.random.default_rng(m)
    tail = list(range(max(0, m - 128), m))
    rest = g.choice(max(1, m - 128), size=min(max(0, count - len(tail)), max(1, m - 128)),
                    replace=False).tolist()
    return sorted(set(tail + rest))


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", CONFIGS)
def test_config_at_full_size(ops, name, mode):
    W = import_pkg("workloads")
    w = W.WORKLOADS[name]
    A, B = W.device_inputs(w)
    op = ops.OPERATORS[w.pid].forward
    with ops.precision(mode):
        C = op(A, B)
        torch.cuda.synchronize()
        C2 = op(A, B)                    # a second call into a fresh output
    torch.cuda.synchronize()
    assert ops.read_device_error(torch.cuda.current_device()) == 0
    assert torch.isfinite(C).all()
    err = full_check(name, A, B, C)
    assert err <= TOL[mode], f"{name} {mode}: full rel_fro {err:.3e} > {TOL[mode]:.0e}"
    assert torch.equal(C, C2) or full_check(name, A, B, C2) <= TOL[mode]
    serr = sample_check(name, A, B, C)
    assert serr <= TOL[mode], f"{name} {mode}: sampled rel_fro {serr:.3e} vs oracle"
    if name in ("upper_tri", "lower_tri"):
        masked = torch.tril(C, -1) if name == "upper_tri" else torch.triu(C, 1)
        assert torch.count_nonzero(masked).item() == 0, "masked triangle must be exactly zero"


@pytest.mark.parametrize("name", ["upper_tri", "lower_tri"])
def test_triangular_full_size_unmasked_inputs(ops, name):
    """K14 masks its own inputs (kernels/14_...:74-75,84-85): unmasked N(0,1)
    operands at N = 4096 give triu(triu(A) triu(B)) (tril for K15's op)."""
    n = 4096
    g = torch.Generator(device="cuda").manual_seed(4096 + len(name))
    A = torch.randn(n, n, generator=g, device="cuda")
    B = torch.randn(n, n, generator=g, device="cuda")
    C = ops.OPERATORS[14 if name == "upper_tri" else 15].forward(A, B)
    torch.cuda.synchronize()
    assert full_check(name, A, B, C) <= TOL["tf32"]
    assert sample_check(name, A, B, C) <= TOL["tf32"]
    masked = torch.tril(C, -1) if name == "upper_tri" else torch.triu(C, 1)
    assert torch.count_nonzero(masked).item() == 0
