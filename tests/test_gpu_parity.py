"""Parity of the CUDA path against the fp64 CPU oracle, on seeded inputs.

Tolerances (relative Frobenius norm against float64): 1e-2 in TF32 mode,
1e-3 in 3xTF32 mode.  Masked triangles must be exactly zero; diag(a).B must
be bit-exact against the fp32 CPU product.  Small and odd shapes exercise
the tails (tiles +-1, K = 1, unaligned pitches that go through the staged
copy, transposed views).
"""
import numpy as np
import pytest
import torch

from conftest import import_pkg
from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = O.TOL


def _randn(g, *shape):
    return torch.randn(*shape, generator=g, dtype=torch.float32)


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _check(got, ref, mode):
    err = O.rel_fro(got.double().cpu().numpy(), ref)
    assert err <= TOL[mode], f"rel_fro {err:.3e} > {TOL[mode]:.0e}"
    return err


MODES = ["tf32", "3xtf32"]

NN_SHAPES = [(1, 1, 1), (1, 7, 3), (127, 65, 33), (128, 256, 32), (129, 257, 31),
             (256, 128, 64), (300, 500, 1), (64, 8, 4096), (1000, 1000, 1000),
             (513, 769, 200), (128, 384, 96)]


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("m,n,k", NN_SHAPES)
def test_standard_nn(ops, mode, m, n, k):
    g = _gen(m * 7919 + n * 31 + k)
    A, B = _randn(g, m, k), _randn(g, k, n)
    with ops.precision(mode):
        C = ops.p2.forward(A.cuda(), B.cuda())
    assert C.shape == (m, n) and C.dtype == torch.float32
    _check(C, O.standard(A.numpy(), B.numpy()), mode)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("pid", [16, 17, 18])
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (128, 256, 64), (130, 70, 33), (1024, 512, 512),
                                   (96, 320, 1000)])
def test_transposed(ops, mode, pid, m, n, k):
    g = _gen(pid * 100003 + m + n + k)
    A = _randn(g, k, m) if pid in (16, 18) else _randn(g, m, k)
    B = _randn(g, n, k) if pid in (17, 18) else _randn(g, k, n)
    with ops.precision(mode):
        C = ops.OPERATORS[pid].forward(A.cuda(), B.cuda())
    assert C.shape == (m, n)
    _check(C, O.BY_PID[pid](A.numpy(), B.numpy()), mode)


def test_reference_names_are_aliases(ops):
    assert ops.p16.matmul_transposed_cuda is ops.p16.forward
    assert ops.p17.matmul_cuda is ops.p17.forward
    assert ops.p12.diag_mult_cuda is ops.p12.forward
    assert ops.p15.lower_tri_mul_cuda is ops.p15.forward
    assert ops.p3.batched_matmul_cuda is ops.p3.forward
    assert ops.p7.gemm_cuda is ops.p7.forward


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("batch,m,n,k", [(1, 64, 64, 64), (3, 130, 70, 40), (8, 256, 512, 128),
                                         (5, 1, 33, 17)])
def test_batched(ops, mode, batch, m, n, k):
    g = _gen(batch * 17 + m)
    A, B = _randn(g, batch, m, k), _randn(g, batch, k, n)
    with ops.precision(mode):
        C = ops.p3.forward(A.cuda(), B.cuda())
    assert C.shape == (batch, m, n)
    _check(C, O.batched(A.numpy(), B.numpy()), mode)


def test_batched_strided_views(ops):
    g = _gen(5)
    base = _randn(g, 4, 200, 96)
    A = base[:, 8:136, :64]              # pitch 96, batch stride 200*96
    B = _randn(g, 4, 64, 80)
    C = ops.p3.forward(A.cuda(), B.cuda())
    _check(C, O.batched(A.numpy(), B.numpy()), "tf32")


@pytest.mark.parametrize("mode", MODES)
def test_tensor3d(ops, mode):
    g = _gen(10)
    A, B = _randn(g, 4, 100, 96), _randn(g, 96, 200)
    with ops.precision(mode):
        C = ops.p10.forward(A.cuda(), B.cuda())
    assert C.shape == (4, 100, 200)
    _check(C, O.tensor3d(A.numpy(), B.numpy()), mode)


@pytest.mark.parametrize("mode", MODES)
def test_tensor4d(ops, mode):
    g = _gen(11)
    A, B = _randn(g, 2, 3, 50, 64), _randn(g, 64, 96)
    with ops.precision(mode):
        C = ops.p11.forward(A.cuda(), B.cuda())
    assert C.shape == (2, 3, 50, 96)
    _check(C, O.tensor4d(A.numpy(), B.numpy()), mode)


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (64, 64), (4096, 4096), (17, 4099),
                                       (1000, 4)])
def test_diag_bit_exact(ops, rows, cols):
    g = _gen(rows + cols)
    a, B = _randn(g, rows), _randn(g, rows, cols)
    out = ops.p12.forward(a.cuda(), B.cuda()).cpu().numpy()
    np.testing.assert_array_equal(out, O.diag(a.numpy(), B.numpy()))


def test_diag_strided_rows(ops):
    g = _gen(3)
    base = _randn(g, 64, 100)
    B = base[:, :96]
    a = _randn(g, 64)
    out = ops.p12.forward(a.cuda(), B.cuda()).cpu().numpy()
    np.testing.assert_array_equal(out, O.diag(a.numpy(), B.numpy()))


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("pid", [14, 15])
@pytest.mark.parametrize("n", [1, 5, 64, 128, 129, 300, 513, 1024])
@pytest.mark.parametrize("pre_masked", [True, False])
def test_triangular(ops, mode, pid, n, pre_masked):
    g = _gen(pid * 1000 + n)
    A, B = _randn(g, n, n), _randn(g, n, n)
    if pre_masked:
        tri = torch.triu if pid == 14 else torch.tril
        A, B = tri(A), tri(B)
    with ops.precision(mode):
        C = ops.OPERATORS[pid].forward(A.cuda(), B.cuda())
    ref = O.BY_PID[pid](A.numpy(), B.numpy())
    _check(C, ref, mode)
    Cc = C.cpu()
    masked = torch.tril(Cc, -1) if pid == 14 else torch.triu(Cc, 1)
    assert torch.count_nonzero(masked).item() == 0, "masked triangle must be exactly zero"


@pytest.mark.parametrize("mode", MODES)
def test_symmetric(ops, mode):
    g = _gen(13)
    X, Y = _randn(g, 384, 384), _randn(g, 384, 384)
    A, B = (X + X.T) / 2, (Y + Y.T) / 2
    with ops.precision(mode):
        C = ops.p13.forward(A.cuda(), B.cuda())
    _check(C, O.symmetric(A.numpy(), B.numpy()), mode)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("m,n,k", [(256, 256, 65536), (128, 96, 20000), (64, 300, 8192)])
def test_split_k(ops, mode, m, n, k):
    g = _gen(k)
    A, B = _randn(g, m, k), _randn(g, k, n)
    with ops.precision(mode):
        C = ops.p6.forward(A.cuda(), B.cuda())
    _check(C, O.large_k(A.numpy(), B.numpy()), mode)


def test_transposed_views_are_read_in_place(ops):
    g = _gen(21)
    At = _randn(g, 200, 150)            # A = At.T is a column-major view
    B = _randn(g, 200, 96)
    C = ops.p2.forward(At.cuda().t(), B.cuda())
    _check(C, O.standard(At.numpy().T, B.numpy()), "tf32")


def test_small_k_and_tall_skinny_semantics(ops):
    g = _gen(22)
    A, B = _randn(g, 1000, 32), _randn(g, 32, 900)
    _check(ops.p7.forward(A.cuda(), B.cuda()), O.small_k(A.numpy(), B.numpy()), "tf32")
    A, B = _randn(g, 700, 64), _randn(g, 64, 700)
    _check(ops.p9.forward(A.cuda(), B.cuda()), O.tall_skinny(A.numpy(), B.numpy()), "tf32")


def test_zero_sizes(ops):
    A = torch.randn(0, 5, device="cuda")
    B = torch.randn(5, 7, device="cuda")
    assert ops.p2.forward(A, B).shape == (0, 7)
    A = torch.randn(6, 0, device="cuda")
    B = torch.randn(0, 7, device="cuda")
    C = ops.p2.forward(A, B)
    assert C.shape == (6, 7) and torch.count_nonzero(C).item() == 0


def test_errors_are_raised_like_torch_check(ops):
    with pytest.raises(RuntimeError, match="inner dimensions"):
        ops.p2.forward(torch.randn(4, 5, device="cuda"), torch.randn(6, 7, device="cuda"))
    with pytest.raises(RuntimeError, match="float32"):
        ops.p2.forward(torch.randn(4, 5, device="cuda").double(),
                       torch.randn(5, 7, device="cuda").double())
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.p2.forward(torch.randn(4, 5), torch.randn(5, 7))
    with pytest.raises(RuntimeError, match="1-dimensional"):
        ops.p12.forward(torch.randn(4, 4, device="cuda"), torch.randn(4, 4, device="cuda"))


def test_capi_direct_call(capi):
    """The C ABI called straight from ctypes with torch-allocated buffers."""
    g = _gen(99)
    A, B = _randn(g, 300, 200).cuda(), _randn(g, 200, 260).cuda()
    C = torch.empty(300, 260, device="cuda")
    d = capi.make_desc(300, 260, 200, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr())
    rc = capi.gemm(d, torch.cuda.current_stream().cuda_stream)
    assert rc == capi.B2G_OK, capi.status_string(rc)
    torch.cuda.synchronize()
    _check(C, O.standard(A.cpu().numpy(), B.cpu().numpy()), "tf32")
    # An unaligned pitch needs workspace: without it the call is refused.
    A2 = _randn(g, 64, 33).cuda()
    B2 = _randn(g, 33, 64).cuda()
    C2 = torch.empty(64, 64, device="cuda")
    d2 = capi.make_desc(64, 64, 33, a=A2.data_ptr(), b=B2.data_ptr(), c=C2.data_ptr())
    assert capi.gemm(d2) == capi.B2G_ERR_WORKSPACE


def test_no_device_errors_recorded(ops):
    torch.cuda.synchronize()
    assert ops.read_device_error(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_batched_matmul_from_host_streams_chunks(ops, chunks):
    g = _gen(77 + chunks)
    A = _randn(g, 10, 130, 96).pin_memory()
    B = _randn(g, 10, 96, 200).pin_memory()
    C = ops.batched_matmul_from_host(A, B, chunks=chunks)
    assert C.shape == (10, 130, 200) and not C.is_cuda
    _check(C, O.batched(A.numpy(), B.numpy()), "tf32")
    ref = ops.p3.forward(A.cuda(), B.cuda()).cpu()
    assert torch.equal(C, ref)


def test_batched_matmul_out_validates_shapes(ops):
    A = torch.randn(2, 8, 4, device="cuda")
    B = torch.randn(2, 4, 6, device="cuda")
    with pytest.raises(RuntimeError, match="C must be"):
        ops.batched_matmul_out(A, B, torch.empty(2, 8, 5, device="cuda"))


@pytest.mark.parametrize("m,k", [(1, 1), (7, 3), (4096, 4096), (100, 100003), (3, 65536),
                                 (20000, 64), (33, 4097)])
def test_gemv(ops, m, k):
    g = _gen(m * 13 + k)
    A, x = _randn(g, m, k), _randn(g, k, 1)
    y = ops.p4.forward(A.cuda(), x.cuda())
    assert y.shape == (m, 1)
    err = O.rel_fro(y.cpu().double().numpy(), O.gemv(A.numpy(), x.numpy()))
    assert err <= 1e-5, err           # fp32 accumulation against fp64


def test_gemv_strided_rows(ops):
    g = _gen(8)
    base = _randn(g, 50, 700)
    A = base[:, 3:603]                 # pitch 700, unaligned start
    x = _randn(g, 600, 1)
    y = ops.p4.gemv_cuda(A.cuda(), x.cuda())
    assert O.rel_fro(y.cpu().double().numpy(), O.gemv(A.numpy(), x.numpy())) <= 1e-5


@pytest.mark.parametrize("shape", [(1,), (3, 5), (4096, 4096), (1000, 1003), (7, 1, 9)])
def test_matrix_scalar_bit_exact(ops, shape):
    g = _gen(len(shape) * 11 + shape[0])
    A = _randn(g, *shape)
    C = ops.p5.matrix_scalar_mult_cuda(A.cuda(), 0.37)
    np.testing.assert_array_equal(C.cpu().numpy(), O.matrix_scalar(A.numpy(), 0.37))


@pytest.mark.parametrize("m,n,k", [(256, 256, 65536), (1024, 2048, 4096), (300, 500, 20000)])
def test_split_k_clears_output_in_kernel(ops, m, n, k):
    """Split-K pieces reduce-add into C; the first piece of each tile clears it
    in the kernel.  C starts as NaN and is written three times in a row."""
    g = _gen(m + n + k)
    A, B = _randn(g, 1, m, k).cuda(), _randn(g, 1, k, n).cuda()
    C = torch.full((1, m, n), float("nan"), device="cuda")
    ref = O.batched(A.cpu().numpy(), B.cpu().numpy())
    for _ in range(3):
        ops.batched_matmul_out(A, B, C)
        torch.cuda.synchronize()
        assert torch.isfinite(C).all()
        _check(C, ref, "tf32")
    assert ops.read_device_error(torch.cuda.current_device()) == 0


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("pid", [14, 15])
@pytest.mark.parametrize("n", [300, 1024, 4096])
@pytest.mark.parametrize("views", ["ta", "tb", "tatb"])
def test_triangular_transposed_views(ops, mode, pid, n, views):
    """Triangular products on transposed operand views (A or B stored
    transposed, read in place): the engine masks the K blocks that the
    diagonal crosses in its transform warps and loads wholly masked boxes as
    zero fill (TF32), or transforms every stage (3xTF32).  Unmasked N(0,1)
    inputs: the operator masks them itself (kernels/14_...:74-75,84-85)."""
    g = _gen(pid * 7 + n + len(views))
    A, B = _randn(g, n, n), _randn(g, n, n)
    Ad = A.t().contiguous().cuda().t() if "ta" in views else A.cuda()
    Bd = B.t().contiguous().cuda().t() if "tb" in views else B.cuda()
    with ops.precision(mode):
        C = ops.OPERATORS[pid].forward(Ad, Bd)
    _check(C, O.BY_PID[pid](A.numpy(), B.numpy()), mode)
    masked = torch.tril(C, -1) if pid == 14 else torch.triu(C, 1)
    assert torch.count_nonzero(masked).item() == 0
    assert ops.read_device_error(torch.cuda.current_device()) == 0


GATE_CHILD = r"""
import importlib, json, sys, torch
sys.path.insert(0, sys.argv[1])
ops = importlib.import_module("cupilot-kernels_b200.ops")
out = []
for pid, n in ((14, 4096), (15, 4096), (14, 1536), (15, 2048)):
    g = torch.Generator(device="cuda").manual_seed(pid + n)
    A = torch.randn(n, n, generator=g, device="cuda")
    B = torch.randn(n, n, generator=g, device="cuda")
    tri = torch.triu if pid == 14 else torch.tril
    ref = tri(tri(A).double() @ tri(B).double())
    C = ops.OPERATORS[pid].forward(A, B)
    masked = torch.tril(C, -1) if pid == 14 else torch.triu(C, 1)
    out.append([float(((C.double() - ref).norm() / ref.norm()).item()),
                int(torch.count_nonzero(masked).item())])
print(json.dumps({"res": out, "code": ops.read_device_error(0)}))
"""


def test_triangular_gated_path_on_untransposed_operands():
    """The in-engine masking (B2G_TRI_PATH=gate, a tuning knob) on the
    untransposed configs, where it runs split tiles cleared in the kernel
    and many units per CTA pair."""
    import json
    import os
    import subprocess
    import sys

    from conftest import REPO

    env = dict(os.environ, B2G_TUNING="1", B2G_TRI_PATH="gate")
    r = subprocess.run([sys.executable, "-c", GATE_CHILD, str(REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["code"] == 0, out
    for err, nz in out["res"]:
        assert err <= 1e-2 and nz == 0, out
