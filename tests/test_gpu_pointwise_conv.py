"""Pointwise (1x1) convolution — kernels/87_conv_pointwise_2D_best_kernel.cu:451.

out (N, Cout, H, W) = sum over Cin of weight[o, c] * input[n, c, h, w] + bias[o],
run as one batched GEMM with the bias added in the epilogue.  Parity against
the fp64 oracle (relative Frobenius 1e-2 TF32, 1e-3 3xTF32), tails on every
dimension, unaligned H*W (staged copy), split-K (the bias must be added once),
in_channels == 0 (bias only), and the reference kernel itself where it is
built and the shape is inside its contract.
"""
import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

MODES = ["tf32", "3xtf32"]

# (batch, in_channels, out_channels, height, width)
SHAPES = [(1, 1, 1, 1, 1), (2, 3, 64, 5, 7), (3, 40, 130, 9, 9), (2, 129, 257, 16, 16),
          (16, 64, 128, 32, 32), (1, 256, 512, 28, 28), (4, 32, 96, 1, 1000)]


def _inputs(seed, n, cin, cout, h, w, bias=True, w4d=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, cin, h, w, generator=g)
    wt = torch.randn(cout, cin, 1, 1, generator=g) if w4d else torch.randn(cout, cin, generator=g)
    b = torch.randn(cout, generator=g) if bias else None
    return x, wt, b


def _check(out, x, wt, b, mode):
    ref = O.pointwise_conv(x.numpy(), wt.numpy(), None if b is None else b.numpy())
    assert tuple(out.shape) == ref.shape and out.dtype == torch.float32
    err = O.rel_fro(out.double().cpu().numpy(), ref)
    assert err <= O.TOL[mode], f"rel_fro {err:.3e} > {O.TOL[mode]:.0e}"


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("bias", [True, False])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_pointwise_conv(ops, mode, bias, shape):
    x, wt, b = _inputs(sum(shape) * 13 + bias, *shape, bias=bias)
    with ops.precision(mode):
        out = ops.p87.forward(x.cuda(), wt.cuda(), None if b is None else b.cuda())
    _check(out, x, wt, b, mode)


def test_reference_name_and_2d_weight(ops):
    x, wt, b = _inputs(5, 2, 48, 64, 8, 8, w4d=False)
    out2 = ops.p87.pointwise_conv_cuda(x.cuda(), wt.cuda(), b.cuda())
    out4 = ops.pointwise_conv(x.cuda(), wt.view(64, 48, 1, 1).cuda(), bias=b.cuda())
    assert torch.equal(out2, out4)
    _check(out2, x, wt, b, "tf32")


@pytest.mark.parametrize("mode", MODES)
def test_split_k_adds_bias_once(ops, mode):
    # Few output tiles and a long channel reduction: the planner splits K and
    # the K pieces reduce-add into C; only the first piece carries the bias.
    x, wt, b = _inputs(6, 1, 16384, 64, 4, 4)
    b = b * 100.0
    with ops.precision(mode):
        out = ops.p87.forward(x.cuda(), wt.cuda(), b.cuda())
    _check(out, x, wt, b, mode)


def test_zero_in_channels_writes_bias(ops):
    x = torch.empty(2, 0, 3, 5, device="cuda")
    wt = torch.empty(4, 0, 1, 1, device="cuda")
    b = torch.arange(4, dtype=torch.float32, device="cuda")
    out = ops.p87.forward(x, wt, b)
    assert torch.equal(out, b.view(1, 4, 1, 1).expand(2, 4, 3, 5))
    assert torch.count_nonzero(ops.p87.forward(x, wt)).item() == 0


def test_zero_sizes_and_errors(ops):
    assert ops.p87.forward(torch.empty(0, 3, 4, 4, device="cuda"),
                           torch.randn(5, 3, 1, 1, device="cuda")).shape == (0, 5, 4, 4)
    with pytest.raises(RuntimeError, match="input channels"):
        ops.p87.forward(torch.randn(1, 3, 4, 4, device="cuda"), torch.randn(5, 4, 1, 1, device="cuda"))
    with pytest.raises(RuntimeError, match="bias"):
        ops.p87.forward(torch.randn(1, 3, 4, 4, device="cuda"), torch.randn(5, 3, 1, 1, device="cuda"),
                        torch.randn(4, device="cuda"))
    with pytest.raises(RuntimeError, match="weight"):
        ops.p87.forward(torch.randn(1, 3, 4, 4, device="cuda"), torch.randn(5, 3, 3, 3, device="cuda"))


def test_capi_direct_call(capi):
    x, wt, b = _inputs(7, 3, 24, 40, 6, 10)
    xd, wd, bd = x.cuda(), wt.cuda(), b.cuda()
    out = torch.empty(3, 40, 6, 10, device="cuda")
    ws = capi.pointwise_conv_workspace_bytes(xd.data_ptr(), wd.data_ptr(), out.data_ptr(),
                                             3, 24, 40, 60)
    assert ws == 0
    rc = capi.pointwise_conv(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), out.data_ptr(),
                             3, 24, 40, 60, stream=torch.cuda.current_stream().cuda_stream)
    assert rc == capi.B2G_OK, capi.status_string(rc)
    torch.cuda.synchronize()
    _check(out, x, wt, b, "tf32")
    # H*W = 35 is not 16-byte aligned: the staged copy needs workspace.
    x2 = torch.randn(2, 8, 5, 7, device="cuda")
    w2 = torch.randn(16, 8, device="cuda")
    o2 = torch.empty(2, 16, 5, 7, device="cuda")
    assert capi.pointwise_conv_workspace_bytes(x2.data_ptr(), w2.data_ptr(), o2.data_ptr(),
                                               2, 8, 16, 35) > 0
    assert capi.pointwise_conv(x2.data_ptr(), w2.data_ptr(), 0, o2.data_ptr(),
                               2, 8, 16, 35) == capi.B2G_ERR_WORKSPACE


def test_matches_reference_kernel(ops):
    """Against the reference's own kernel (compiled from kernels/87_*.cu), on a
    shape inside its contract: Cout % 128 == 0, Cin % 8 == 0, H*W % 64 == 0."""
    try:
        from oracle import build_ref
        ref_f = build_ref.load(87)
    except ImportError as e:
        pytest.skip(str(e))
    x, wt, b = _inputs(8, 4, 64, 256, 32, 32)
    xd, wd, bd = x.cuda(), wt.cuda(), b.cuda()
    ref = ref_f(xd, wd, bd)
    with ops.precision("3xtf32"):
        out = ops.p87.forward(xd, wd, bd)
    err = O.rel_fro(out.double().cpu().numpy(), ref.double().cpu().numpy())
    assert err <= 1e-3, f"rel_fro vs reference kernel {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_and_bfloat16_inputs(ops, dtype):
    """fp16 / bf16 in, same dtype out (as the reference's dispatch returns)."""
    x, wt, b = _inputs(11, 2, 32, 64, 8, 8)
    x, wt, b = x.to(dtype), wt.to(dtype), b.to(dtype)
    out = ops.p87.forward(x.cuda(), wt.cuda(), b.cuda())
    assert out.dtype == dtype and out.shape == (2, 64, 8, 8)
    ref = O.pointwise_conv(x.float().numpy(), wt.float().numpy(), b.float().numpy())
    tol = 1e-2 if dtype == torch.float16 else 2e-2   # output rounding of the narrow type
    assert O.rel_fro(out.double().cpu().numpy(), ref) <= tol
