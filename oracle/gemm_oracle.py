"""CPU oracle for the fp32-input GEMM family — TEST INFRASTRUCTURE ONLY.

A restatement, in float64 numpy, of what each reference operator computes.
It is the parity checker for the CUDA path (tests/, smoke(), bench.py's
cpu_baseline leg); nothing in the product imports it.

Pinning: the reference (champloo2878/cuPilot-Kernels) ships no tests, golden
vectors or fixtures for this path, so there is nothing of the reference's own
to pin against on the CPU.  This oracle is pinned instead by closed-form
known answers (tests/golden/known_answers.json, made by
tests/golden/make_known_answers.py from formulas, not from this module) and,
on the GPU box, by the reference kernels themselves compiled from
kernels/*.cu (oracle/build_ref.py), whose outputs must agree with this oracle
within their fp16/bf16 operand rounding.

Operator semantics (reference file:line):
  square / standard / large-K / small-K / irregular / tall-skinny: C = A B
      kernels/1_...:189, 2_...:117, 6_...:128, 7_...:80, 8_...:155, 9_...:145
  batched: C[b] = A[b] B[b]                         kernels/3_...:113
  3-D:  out[n] = A[n] B  (A (n,m,k), B (k,l))       kernels/10_...:180
  4-D:  einsum('bijl,lk->bijk')                     kernels/11_...:132, view at :165
  diag: out = a[:, None] * B  (a 1-D)               kernels/12_...:9-38
  symmetric: C = A B (symmetry not required)        kernels/13_...:134
  upper: C = triu(triu(A) triu(B))  (K14 masks its inputs, :74-75, :84-85,
         and its output store, :122-128)            kernels/14_...:135
  lower: C = tril(tril(A) tril(B))  (K15 assumes lower inputs, masks the
         output, :53-66, :117-146)                  kernels/15_...:155
  A^T B (A stored (K,M))                            kernels/16_...:124
  A B^T (B stored (N,K))                            kernels/17_...:267
  A^T B^T                                           kernels/18_...:152
  pointwise conv: out[n,o,h,w] = sum_c W[o,c] x[n,c,h,w] + bias[o]
         (K87 accumulates over in_channels, :340, then adds the bias,
         :374-386)                                  kernels/87_...:451
  attention: out = softmax(Q K^T / sqrt(D)) V per (batch, head), fp16 in
         and out (K97 scales by 1/sqrt(embed_dim), :266, takes the row max,
         exponentials and their sum, :41-89, then weights V, :205-224)
                                                    kernels/97_...:256
"""
from __future__ import annotations

import numpy as np


def _f64(x):
    return np.asarray(x, dtype=np.float64)


def gemv(A, B):
    """C (M, 1) = A (M, K) . B (K, 1)          kernels/4_...:84"""
    return _f64(A) @ _f64(B)


def matrix_scalar(A, s):
    """C = A * s in fp32, one rounding per element   kernels/5_...:47"""
    return (np.asarray(A, dtype=np.float32) * np.float32(s)).astype(np.float32)


def matmul(A, B):
    return _f64(A) @ _f64(B)


def square(A, B):
    return matmul(A, B)


standard = large_k = small_k = irregular = tall_skinny = symmetric = square


def batched(A, B):
    return np.matmul(_f64(A), _f64(B))


def tensor3d(A, B):
    return np.matmul(_f64(A), _f64(B))


def tensor4d(A, B):
    A = _f64(A)
    b, i, j, l = A.shape
    return (A.reshape(b * i * j, l) @ _f64(B)).reshape(b, i, j, B.shape[1])


def diag(a, B):
    """Exactly one fp32 rounding per element, as the kernel's single multiply."""
    a = np.asarray(a, dtype=np.float32)
    B = np.asarray(B, dtype=np.float32)
    return (a[:, None] * B).astype(np.float32)


def upper_tri(A, B):
    return np.triu(np.triu(_f64(A)) @ np.triu(_f64(B)))


def lower_tri(A, B):
    return np.tril(np.tril(_f64(A)) @ np.tril(_f64(B)))


def transposed_a(A, B):
    return _f64(A).T @ _f64(B)


def transposed_b(A, B):
    return _f64(A) @ _f64(B).T


def transposed_both(A, B):
    return _f64(A).T @ _f64(B).T


def pointwise_conv(x, weight, bias=None):
    """out (N, Cout, H, W) = 1x1 conv of x (N, Cin, H, W)   kernels/87_...:451

    weight is (Cout, Cin) or (Cout, Cin, 1, 1); bias (Cout,) or None.
    """
    x = _f64(x)
    w = _f64(weight).reshape(weight.shape[0], -1)
    n, c, h, wd = x.shape
    out = np.einsum("oc,ncs->nos", w, x.reshape(n, c, h * wd))
    if bias is not None:
        out = out + _f64(bias).reshape(1, -1, 1)
    return out.reshape(n, w.shape[0], h, wd)


def sdpa(Q, K, V):
    """out (B, H, S, D) = softmax(Q K^T / sqrt(D)) V in float64   kernels/97_...:256"""
    q, k, v = _f64(Q), _f64(K), _f64(V)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) / np.sqrt(q.shape[-1])
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


BY_PID = {
    4: gemv, 5: matrix_scalar,
    1: square, 2: standard, 3: batched, 6: large_k, 7: small_k, 8: irregular,
    9: tall_skinny, 10: tensor3d, 11: tensor4d, 12: diag, 13: symmetric,
    14: upper_tri, 15: lower_tri, 16: transposed_a, 17: transposed_b, 18: transposed_both,
    87: pointwise_conv, 97: sdpa,
}


def rel_fro(x, ref) -> float:
    """||x - ref||_F / ||ref||_F in float64 (0 when both are zero)."""
    x = _f64(x)
    ref = _f64(ref)
    den = np.linalg.norm(ref.ravel())
    num = np.linalg.norm((x - ref).ravel())
    if den == 0.0:
        return float(num)
    return float(num / den)


# Relative-Frobenius tolerances per precision mode.
TOL = {"tf32": 1e-2, "3xtf32": 1e-3}
