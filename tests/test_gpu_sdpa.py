"""Scaled-dot-product attention — kernels/97_ScaledDotProductAttention_best_kernel.cu:256.

out = softmax(Q K^T / sqrt(D)) V for fp16 (batch, heads, seq, dim) tensors,
against the float64 oracle on the same fp16 inputs.  Tolerance: relative
Frobenius 5e-3 (the result is rounded to fp16, and P enters the second
product as fp16).  Tails: seq not a multiple of the 128-row query block or
of the 64-key slice, dim not a multiple of the 256-column output chunk, a
single key; peaked softmax rows; the reference kernel itself at its own
contract (seq 512, dim 1024).
"""
import numpy as np
import pytest
import torch

from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu

TOL = 5e-3

SHAPES = [(1, 1, 1, 64), (1, 2, 37, 64), (2, 3, 128, 128), (1, 2, 200, 192), (2, 2, 300, 320),
          (1, 1, 512, 1024), (2, 3, 511, 256), (1, 2, 257, 512)]


def _inputs(seed, b, h, s, d, q_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(b, h, s, d, generator=g) * q_scale).half()
    k = torch.randn(b, h, s, d, generator=g).half()
    v = torch.randn(b, h, s, d, generator=g).half()
    return q, k, v


def _check(out, q, k, v, tol=TOL):
    ref = O.sdpa(q.numpy(), k.numpy(), v.numpy())
    assert tuple(out.shape) == ref.shape and out.dtype == torch.float16
    err = O.rel_fro(out.double().cpu().numpy(), ref)
    assert err <= tol, f"rel_fro {err:.3e} > {tol:.0e}"
    return err


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_sdpa_matches_oracle(ops, shape):
    q, k, v = _inputs(sum(shape), *shape)
    out = ops.p97.forward(q.cuda(), k.cuda(), v.cuda())
    _check(out, q, k, v)


def test_peaked_rows(ops):
    # Large logits: the row max must be subtracted before the exponentials.
    q, k, v = _inputs(3, 1, 2, 256, 128, q_scale=8.0)
    out = ops.p97.fused_attention_cuda(q.cuda(), k.cuda(), v.cuda())
    assert torch.isfinite(out).all()
    _check(out, q, k, v)


def test_rows_of_one_key_copy_v(ops):
    q, k, v = _inputs(4, 2, 2, 1, 64)
    out = ops.p97.forward(q.cuda(), k.cuda(), v.cuda())
    assert torch.equal(out.cpu(), v)


def test_errors(ops):
    x = torch.randn(1, 1, 8, 64, device="cuda")
    with pytest.raises(RuntimeError, match="float16"):
        ops.p97.forward(x, x, x)
    y = torch.randn(1, 1, 513, 64, device="cuda").half()
    with pytest.raises(RuntimeError, match="512"):
        ops.p97.forward(y, y, y)
    z = torch.randn(1, 1, 8, 96, device="cuda").half()
    with pytest.raises(RuntimeError, match="multiple of 64"):
        ops.p97.forward(z, z, z)
    e = torch.empty(0, 2, 8, 64, device="cuda").half()
    assert ops.p97.forward(e, e, e).shape == e.shape


def test_no_device_error(ops):
    torch.cuda.synchronize()
    assert ops.read_device_error(torch.cuda.current_device()) == 0


def test_matches_reference_kernel(ops):
    """Against the reference's own kernel (kernels/97_*.cu) inside its contract."""
    try:
        from oracle import build_ref
        ref_f = build_ref.load(97)
    except ImportError as e:
        pytest.skip(str(e))
    q, k, v = _inputs(9, 2, 2, 512, 1024)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    ref = ref_f(qd, kd, vd).double().cpu().numpy()
    out = ops.p97.forward(qd, kd, vd).double().cpu().numpy()
    assert O.rel_fro(out, ref) <= TOL
    assert O.rel_fro(ref, O.sdpa(q.numpy(), k.numpy(), v.numpy())) <= TOL
