"""Per-operator entry points mirroring the reference's Part-3 host functions.

The reference builds one JIT module per kernel file, each exporting a single
`torch::Tensor <name>(torch::Tensor A, torch::Tensor B)`.  Here every
operator is an object with `forward(A, B)` and an attribute carrying the
reference's own function name, so both call styles drop in:

    from cupilot_kernels_b200 import ops          # (package dir: cupilot-kernels_b200)
    C = ops.p16.forward(A, B)                      # C = A^T B
    C = ops.p16.matmul_transposed_cuda(A, B)       # same function

Inputs: CUDA float32 tensors (A, B as the reference takes them).  Output:
a new float32 tensor on the same device, produced on the current stream.
Errors raise RuntimeError from TORCH_CHECK, as the reference's TORCH_CHECKs do.

Precision: TF32 by default (`set_precision("3xtf32")` or the
`precision("3xtf32")` context manager selects the split 3xTF32 mode).
"""
from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass
from typing import Callable

from . import native

_ext = native()

PRECISIONS = {"tf32": 0, "3xtf32": 1}


def set_precision(mode: str) -> None:
    """Select the process-wide default: 'tf32' (one TF32 product) or
    '3xtf32' (split, ~fp32 accuracy).  Threads inside a `precision()` block
    keep their own mode."""
    if mode not in PRECISIONS:
        raise ValueError(f"precision must be one of {sorted(PRECISIONS)}, got {mode!r}")
    _ext.set_precision(PRECISIONS[mode])


def get_precision() -> str:
    """The mode this thread's calls use (its override, else the default)."""
    v = _ext.get_precision()
    return next(k for k, i in PRECISIONS.items() if i == v)


@contextlib.contextmanager
def precision(mode: str):
    """Run the block's calls in `mode`, in this thread only."""
    if mode not in PRECISIONS:
        raise ValueError(f"precision must be one of {sorted(PRECISIONS)}, got {mode!r}")
    prev = _ext.get_thread_precision()
    _ext.set_thread_precision(PRECISIONS[mode])
    try:
        yield
    finally:
        _ext.set_thread_precision(prev)


if os.environ.get("B2G_PRECISION"):
    set_precision(os.environ["B2G_PRECISION"].lower())


@dataclass(frozen=True)
class Operator:
    pid: int
    name: str
    ref_name: str           # the reference's Part-3 function name
    ref_site: str           # reference file:line of that function
    forward: Callable

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def __getattr__(self, item):
        if item == self.ref_name:
            return self.forward
        raise AttributeError(item)


_K = "kernels/"
OPERATORS = {
    4: Operator(4, "gemv", "gemv_cuda",
                _K + "4_Matrix_vector_multiplication_best_kernel.cu:84", _ext.gemv),
    5: Operator(5, "matrix_scalar", "matrix_scalar_mult_cuda",
                _K + "5_Matrix_scalar_multiplication_best_kernel.cu:47", _ext.matrix_scalar_mult),
    1: Operator(1, "square", "matmul_cuda",
                _K + "1_Square_matrix_multiplication_best_kernel.cu:189", _ext.square_matmul),
    2: Operator(2, "standard", "matmul_cuda",
                _K + "2_Standard_matrix_multiplication_best_kernel.cu:117", _ext.standard_matmul),
    3: Operator(3, "batched", "batched_matmul_cuda",
                _K + "3_Batched_matrix_multiplication_best_kernel.cu:113", _ext.batched_matmul),
    6: Operator(6, "large_k", "matmul_cuda",
                _K + "6_Matmul_with_large_K_dimension_best_kernel.cu:128", _ext.large_k_matmul),
    7: Operator(7, "small_k", "gemm_cuda",
                _K + "7_Matmul_with_small_K_dimension_best_kernel.cu:80", _ext.small_k_matmul),
    8: Operator(8, "irregular", "matmul_cuda",
                _K + "8_Matmul_with_irregular_shapes_best_kernel.cu:155", _ext.irregular_matmul),
    9: Operator(9, "tall_skinny", "tall_skinny_matmul_cuda",
                _K + "9_Tall_skinny_matrix_multiplication_best_kernel.cu:145",
                _ext.tall_skinny_matmul),
    10: Operator(10, "tensor3d", "batched_matmul_cuda",
                 _K + "10_3D_tensor_matrix_multiplication_best_kernel.cu:180",
                 _ext.tensor3d_matmul),
    11: Operator(11, "tensor4d", "tensor_matmul_cuda",
                 _K + "11_4D_tensor_matrix_multiplication_best_kernel.cu:132",
                 _ext.tensor4d_matmul),
    12: Operator(12, "diag", "diag_mult_cuda",
                 _K + "12_Matmul_with_diagonal_matrices_best_kernel.cu:43", _ext.diag_matmul),
    13: Operator(13, "symmetric", "symmetric_matmul_cuda",
                 _K + "13_Matmul_for_symmetric_matrices_best_kernel.cu:134",
                 _ext.symmetric_matmul),
    14: Operator(14, "upper_tri", "upper_tri_matmul_cuda",
                 _K + "14_Matmul_for_upper_triangular_matrices_best_kernel.cu:135",
                 _ext.upper_tri_matmul),
    15: Operator(15, "lower_tri", "lower_tri_mul_cuda",
                 _K + "15_Matmul_for_lower_triangular_matrices_best_kernel.cu:155",
                 _ext.lower_tri_matmul),
    16: Operator(16, "transposed_a", "matmul_transposed_cuda",
                 _K + "16_Matmul_with_transposed_A_best_kernel.cu:124",
                 _ext.matmul_transposed_a),
    17: Operator(17, "transposed_b", "matmul_cuda",
                 _K + "17_Matmul_with_transposed_B_best_kernel.cu:267",
                 _ext.matmul_transposed_b),
    18: Operator(18, "transposed_both", "matmul_transposed_cuda",
                 _K + "18_Matmul_with_transposed_both_best_kernel.cu:152",
                 _ext.matmul_transposed_both),
    # forward(input, weight, bias=None): NCHW 1x1 convolution as a batched GEMM
    87: Operator(87, "pointwise_conv", "pointwise_conv_cuda",
                 _K + "87_conv_pointwise_2D_best_kernel.cu:451", _ext.pointwise_conv),
    # forward(Q, K, V): fp16 attention, (batch, heads, seq <= 512, dim % 64 == 0)
    97: Operator(97, "sdpa", "fused_attention_cuda",
                 _K + "97_ScaledDotProductAttention_best_kernel.cu:256", _ext.fused_attention),
}

for _pid, _op in OPERATORS.items():
    globals()[f"p{_pid}"] = _op
    globals()[_op.name] = _op

gemm = _ext.gemm
read_device_error = _ext.read_device_error


batched_matmul_out = _ext.batched_matmul_out

_HOST_STREAMS = {}


def _host_streams(device):
    key = torch_device_index(device)
    if key not in _HOST_STREAMS:
        import torch

        with torch.cuda.device(key):
            _HOST_STREAMS[key] = (torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream())
    return _HOST_STREAMS[key]


_HOST_BUFFERS = {}


def _host_buffers(dev, sa, sb, sc):
    """Device staging for batched_matmul_from_host, kept per device and grown
    on demand: back-to-back calls reuse it instead of allocating ~2 GB each
    time (the upload stream is ordered after the previous call's downloads)."""
    import math

    import torch

    na, nb, nc = math.prod(sa), math.prod(sb), math.prod(sc)
    # 256-byte aligned sub-buffers (64 floats)
    pa, pb = (na + 63) // 64 * 64, (nb + 63) // 64 * 64
    need = pa + pb + nc
    buf = _HOST_BUFFERS.get(dev.index)
    if buf is None or buf.numel() < need:
        _HOST_BUFFERS[dev.index] = None
        buf = torch.empty(need, dtype=torch.float32, device=dev)
        _HOST_BUFFERS[dev.index] = buf
    return (buf[:na].view(sa), buf[pa:pa + nb].view(sb), buf[pa + pb:pa + pb + nc].view(sc))


def torch_device_index(device):
    import torch

    d = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    return d.index if d.index is not None else torch.cuda.current_device()


def batched_matmul_from_host(A_h, B_h, out=None, chunks=8, device=None, synchronize=True):
    """C = A @ B (batched, fp32) for host tensors, streamed through one GPU.

    The batch is cut into `chunks` pieces; on three CUDA streams the upload
    of piece i+1, the GEMM of piece i and the download of piece i-1 run at
    the same time, so PCIe is busy in both directions while the tensor cores
    work.  A_h (batch, M, K) and B_h (batch, K, N) should be pinned for the
    copies to be asynchronous; `out` (batch, M, N), pinned host memory, is
    allocated when not given.  The caller's current stream is made to wait
    for the last download; with synchronize=True (default) the call also
    blocks until `out` holds the result, otherwise synchronise the current
    stream before reading `out`.
    """
    import torch

    if A_h.dim() != 3 or B_h.dim() != 3 or A_h.shape[0] != B_h.shape[0] \
            or A_h.shape[2] != B_h.shape[1]:
        raise ValueError(f"bmm shape mismatch: {tuple(A_h.shape)} x {tuple(B_h.shape)}")
    if A_h.dtype != torch.float32 or B_h.dtype != torch.float32:
        raise TypeError("A and B must be float32")
    bs, M, K = A_h.shape
    N = B_h.shape[2]
    dev = torch.device("cuda", torch_device_index(device))
    if out is None:
        out = torch.empty(bs, M, N, dtype=torch.float32, pin_memory=True)
    if bs == 0:
        return out
    s_in, s_mm, s_out = _host_streams(dev)
    A_d, B_d, C_d = _host_buffers(dev, (bs, M, K), (bs, K, N), (bs, M, N))
    step = max(1, (bs + chunks - 1) // chunks)
    pieces = [(b0, min(bs, b0 + step)) for b0 in range(0, bs, step)]
    cur = torch.cuda.current_stream(dev)
    for s in (s_in, s_mm, s_out):
        s.wait_stream(cur)
    s_in.wait_stream(s_out)   # the previous call's downloads are done with the buffers
    for b0, b1 in pieces:
        with torch.cuda.stream(s_in):
            A_d[b0:b1].copy_(A_h[b0:b1], non_blocking=True)
            B_d[b0:b1].copy_(B_h[b0:b1], non_blocking=True)
        s_mm.wait_stream(s_in)
        with torch.cuda.stream(s_mm):
            batched_matmul_out(A_d[b0:b1], B_d[b0:b1], C_d[b0:b1])
        s_out.wait_stream(s_mm)
        with torch.cuda.stream(s_out):
            out[b0:b1].copy_(C_d[b0:b1], non_blocking=True)
    cur.wait_stream(s_out)
    if synchronize:
        s_out.synchronize()
    return out
