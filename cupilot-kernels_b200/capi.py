"""ctypes binding of the C ABI in include/b2g_gemm.h.

This is the same binding a non-Torch host would write (cgo / JNI / N-API
stubs look alike): plain structs, pointers and sizes.  Device pointers and
streams are passed as integers (e.g. `tensor.data_ptr()`,
`torch.cuda.current_stream().cuda_stream`).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

from . import LIB_PATH

B2G_OK = 0
B2G_ERR_INVALID_ARG = 1
B2G_ERR_UNSUPPORTED = 2
B2G_ERR_WORKSPACE = 3
B2G_ERR_LAUNCH = 4
B2G_ERR_DEVICE_TIMEOUT = 5
B2G_ERR_NO_DEVICE = 6
B2G_ERR_SCRATCH_LIMIT = 7
NOALLOC_SCRATCH_BYTES = 16 << 20

OP_GEMM, OP_TRI_UPPER, OP_TRI_LOWER = 0, 1, 2
PREC_TF32, PREC_3XTF32 = 0, 1


class GemmDesc(C.Structure):
    _fields_ = [
        ("op", C.c_int32), ("precision", C.c_int32),
        ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64), ("batch", C.c_int64),
        ("a", C.c_void_p), ("lda", C.c_int64), ("stride_a", C.c_int64), ("trans_a", C.c_int32),
        ("b", C.c_void_p), ("ldb", C.c_int64), ("stride_b", C.c_int64), ("trans_b", C.c_int32),
        ("c", C.c_void_p), ("ldc", C.c_int64), ("stride_c", C.c_int64),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_int64),
    ]


class IpcHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]


PEER_MAX_RANKS = 16


class GemmPlan(C.Structure):
    _fields_ = [
        ("block_m", C.c_int32), ("block_n", C.c_int32), ("block_k", C.c_int32),
        ("stages", C.c_int32), ("tiles_m", C.c_int32), ("tiles_n", C.c_int32),
        ("splits", C.c_int32), ("kb_per_split", C.c_int32), ("grid", C.c_int32),
        ("stage_a", C.c_int32), ("stage_b", C.c_int32),
        ("a_mn_major", C.c_int32), ("b_mn_major", C.c_int32),
        ("cluster_ctas", C.c_int32), ("tma_store", C.c_int32), ("tri_diag", C.c_int32),
        ("x3_split", C.c_int32),
        ("work_units", C.c_int64), ("workspace_bytes", C.c_int64),
    ]


_lib = None


def lib(path: Path | None = None) -> C.CDLL:
    """Load libb2g_sm100.so (no GPU needed to load it or to plan)."""
    global _lib
    if _lib is None or path is not None:
        h = C.CDLL(str(path or LIB_PATH))
        h.b2g_gemm_plan_for.argtypes = [C.POINTER(GemmDesc), C.c_int, C.POINTER(GemmPlan)]
        h.b2g_gemm_plan_for.restype = C.c_int
        h.b2g_gemm_workspace_bytes.argtypes = [C.POINTER(GemmDesc)]
        h.b2g_gemm_workspace_bytes.restype = C.c_int64
        h.b2g_gemm.argtypes = [C.POINTER(GemmDesc), C.c_void_p]
        h.b2g_gemm.restype = C.c_int
        h.b2g_gemm_noalloc.argtypes = [C.POINTER(GemmDesc), C.c_void_p]
        h.b2g_gemm_noalloc.restype = C.c_int
        h.b2g_noalloc_read_error.argtypes = [C.c_int, C.POINTER(C.c_int32)]
        h.b2g_noalloc_read_error.restype = C.c_int
        h.b2g_rowscale.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                   C.c_int64, C.c_int64, C.c_void_p]
        h.b2g_rowscale.restype = C.c_int
        h.b2g_gemv.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64,
                               C.c_int64, C.c_void_p]
        h.b2g_gemv.restype = C.c_int
        h.b2g_scale.argtypes = [C.c_void_p, C.c_float, C.c_void_p, C.c_int64, C.c_void_p]
        h.b2g_scale.restype = C.c_int
        h.b2g_pointwise_conv_workspace_bytes.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p,
                                                         C.c_int64, C.c_int64, C.c_int64,
                                                         C.c_int64, C.c_int]
        h.b2g_pointwise_conv_workspace_bytes.restype = C.c_int64
        h.b2g_pointwise_conv.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_int64, C.c_int64, C.c_int64, C.c_int64, C.c_int,
                                         C.c_void_p, C.c_int64, C.c_void_p]
        h.b2g_pointwise_conv.restype = C.c_int
        h.b2g_peer_mailbox_bytes.argtypes = [C.c_int64, C.c_int]
        h.b2g_peer_mailbox_bytes.restype = C.c_int64
        h.b2g_peer_mailbox_create.argtypes = [C.c_int64, C.c_int, C.POINTER(C.c_void_p),
                                              C.POINTER(IpcHandle)]
        h.b2g_peer_mailbox_create.restype = C.c_int
        h.b2g_peer_mailbox_open.argtypes = [C.POINTER(IpcHandle), C.POINTER(C.c_void_p)]
        h.b2g_peer_mailbox_open.restype = C.c_int
        h.b2g_peer_mailbox_close.argtypes = [C.c_void_p]
        h.b2g_peer_mailbox_close.restype = C.c_int
        h.b2g_peer_mailbox_destroy.argtypes = [C.c_void_p]
        h.b2g_peer_mailbox_destroy.restype = C.c_int
        h.b2g_splitk_peer_reduce.argtypes = [C.c_void_p, C.c_void_p, C.c_int64,
                                             C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_int,
                                             C.c_int64, C.c_void_p]
        h.b2g_splitk_peer_reduce.restype = C.c_int
        h.b2g_gemm_splitk_peer.argtypes = [C.POINTER(GemmDesc), C.POINTER(C.c_void_p), C.c_int,
                                           C.c_int, C.c_int, C.c_int64, C.c_void_p]
        h.b2g_gemm_splitk_peer.restype = C.c_int
        h.b2g_read_device_error.argtypes = [C.c_int, C.POINTER(C.c_int32)]
        h.b2g_read_device_error.restype = C.c_int
        h.b2g_status_string.argtypes = [C.c_int]
        h.b2g_status_string.restype = C.c_char_p
        h.b2g_version.argtypes = []
        h.b2g_version.restype = C.c_int
        if path is None:
            _lib = h
        return h
    return _lib


def make_desc(m, n, k, *, a=0, lda=None, b=0, ldb=None, c=0, ldc=None, batch=1, stride_a=0,
              stride_b=0, stride_c=0, trans_a=0, trans_b=0, op=OP_GEMM, precision=PREC_TF32,
              workspace=0, workspace_bytes=0) -> GemmDesc:
    if lda is None:
        lda = m if trans_a else k
    if ldb is None:
        ldb = k if trans_b else n
    if ldc is None:
        ldc = n
    return GemmDesc(op, precision, m, n, k, batch, a, lda, stride_a, trans_a, b, ldb, stride_b,
                    trans_b, c, ldc, stride_c, workspace, workspace_bytes)


def plan(desc: GemmDesc, num_sms: int = 148) -> GemmPlan:
    p = GemmPlan()
    rc = lib().b2g_gemm_plan_for(C.byref(desc), num_sms, C.byref(p))
    if rc != B2G_OK:
        raise ValueError(f"b2g_gemm_plan_for: {status_string(rc)} ({rc})")
    return p


def gemm(desc: GemmDesc, stream: int = 0) -> int:
    return lib().b2g_gemm(C.byref(desc), C.c_void_p(stream))


def gemm_noalloc(desc: GemmDesc, stream: int = 0) -> int:
    """b2g_gemm without any device allocation (fixed 16 MiB staging scratch)."""
    return lib().b2g_gemm_noalloc(C.byref(desc), C.c_void_p(stream))


def noalloc_read_error(device: int = 0) -> int:
    """Read and clear b2g_gemm_noalloc's device error word (0: no wait gave up)."""
    code = C.c_int32(0)
    rc = lib().b2g_noalloc_read_error(device, C.byref(code))
    if rc != B2G_OK:
        raise RuntimeError(f"b2g_noalloc_read_error: {status_string(rc)}")
    return code.value


def rowscale(d, b, out, rows, cols, ldb, ldo, stream: int = 0) -> int:
    return lib().b2g_rowscale(d, b, out, rows, cols, ldb, ldo, C.c_void_p(stream))


def pointwise_conv_workspace_bytes(inp, weight, out, batch, cin, cout, spatial,
                                   precision=PREC_TF32) -> int:
    return lib().b2g_pointwise_conv_workspace_bytes(inp, weight, out, batch, cin, cout, spatial,
                                                    precision)


def pointwise_conv(inp, weight, bias, out, batch, cin, cout, spatial, precision=PREC_TF32,
                   workspace=0, workspace_bytes=0, stream: int = 0) -> int:
    """out[n] = weight . in[n] (+ bias per output channel), NCHW with H*W = spatial."""
    return lib().b2g_pointwise_conv(inp, weight, bias, out, batch, cin, cout, spatial, precision,
                                    workspace, workspace_bytes, C.c_void_p(stream))


def _check(rc, what):
    if rc != B2G_OK:
        raise RuntimeError(f"{what}: {status_string(rc)} ({rc})")


def peer_mailbox_bytes(elems: int, world: int) -> int:
    return lib().b2g_peer_mailbox_bytes(elems, world)


def peer_mailbox_create(elems: int, world: int):
    """Create this rank's mailbox on the current device: (pointer, handle bytes)."""
    ptr, h = C.c_void_p(), IpcHandle()
    _check(lib().b2g_peer_mailbox_create(elems, world, C.byref(ptr), C.byref(h)),
           "b2g_peer_mailbox_create")
    return ptr.value, bytes(h.bytes)


def peer_mailbox_open(handle: bytes) -> int:
    h = IpcHandle()
    C.memmove(h.bytes, handle, 64)
    ptr = C.c_void_p()
    _check(lib().b2g_peer_mailbox_open(C.byref(h), C.byref(ptr)), "b2g_peer_mailbox_open")
    return ptr.value


def peer_mailbox_close(ptr: int) -> None:
    _check(lib().b2g_peer_mailbox_close(ptr), "b2g_peer_mailbox_close")


def peer_mailbox_destroy(ptr: int) -> None:
    _check(lib().b2g_peer_mailbox_destroy(ptr), "b2g_peer_mailbox_destroy")


def splitk_peer_reduce(partial: int, out: int, elems: int, mailboxes, rank: int, root: int,
                       epoch: int, stream: int = 0) -> int:
    arr = (C.c_void_p * len(mailboxes))(*mailboxes)
    return lib().b2g_splitk_peer_reduce(partial, out, elems, arr, len(mailboxes), rank, root,
                                        epoch, C.c_void_p(stream))


def gemm_splitk_peer(desc: GemmDesc, mailboxes, rank: int, root: int, epoch: int,
                     stream: int = 0) -> int:
    arr = (C.c_void_p * len(mailboxes))(*mailboxes)
    return lib().b2g_gemm_splitk_peer(C.byref(desc), arr, len(mailboxes), rank, root, epoch,
                                      C.c_void_p(stream))


def torch_splitk_peer_reduce(t, mailboxes, rank, root, epoch):
    """b2g_splitk_peer_reduce through the Torch extension (no ctypes
    conversion per call): t is the root's output or another rank's partial."""
    from . import native

    native().splitk_peer_reduce(t, list(mailboxes), rank, root, epoch)


def torch_gemm_splitk_peer(A, B, mailboxes, rank, root, epoch):
    """b2g_gemm_splitk_peer through the Torch extension: A, B this rank's
    K slices; returns C (the sum on the root, the partial elsewhere)."""
    from . import native

    return native().splitk_peer_matmul(A, B, list(mailboxes), rank, root, epoch)


def read_device_error(device: int = 0) -> int:
    code = C.c_int32(0)
    rc = lib().b2g_read_device_error(device, C.byref(code))
    if rc != B2G_OK:
        raise RuntimeError(f"b2g_read_device_error: {status_string(rc)}")
    return code.value


def status_string(rc: int) -> str:
    return lib().b2g_status_string(rc).decode()
