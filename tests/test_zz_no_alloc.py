"""b2g_gemm_noalloc: the GEMM entry point for callers that cannot allocate.

Some hosts give this library only their input and output buffers and no way
to allocate device memory (a serving runtime whose pool already owns the
GPU's free memory; a latency-bound loop that cannot pay for cudaMalloc's
possible device synchronisation).  b2g_gemm_noalloc puts everything b2g_gemm
would put in caller workspace or keep in its own device caches (staged
copies of unaligned operands, the 3xTF32 lo parts, the triangular unit
table) in a
fixed 16 MiB file-scope device array instead.  These tests call it through
the C ABI and check its output against the existing b2g_gemm entry point's
(and the fp64 oracle), on two calls in a row (the second call reuses the
array the first one left behind).  Its bounded-wait timeouts are reported
through b2g_noalloc_read_error, which allocates nothing either.

This file is named to be collected last, so that a run stopping at the
first failure has already run every other test.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import REPO
from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(seed, m, n, k, op):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(m, k, generator=g)
    B = torch.randn(k, n, generator=g)
    if op == 1:
        A, B = torch.triu(A), torch.triu(B)
    return A.cuda(), B.cuda()


def _oracle(A, B, op):
    f = {0: O.standard, 1: O.upper_tri, 2: O.lower_tri}[op]
    return f(A.cpu().numpy(), B.cpu().numpy())


def _with_workspace(capi, A, B, m, n, k, op, prec, stream):
    """The existing entry point, with caller-allocated workspace."""
    C = torch.empty(m, n, device="cuda")
    d = capi.make_desc(m, n, k, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr(), op=op,
                       precision=prec)
    ws_bytes = capi.lib().b2g_gemm_workspace_bytes(d)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    d.workspace, d.workspace_bytes = ws.data_ptr(), ws_bytes
    rc = capi.gemm(d, stream)
    assert rc == capi.B2G_OK, capi.status_string(rc)
    torch.cuda.synchronize()
    return C, ws_bytes


def _noalloc_twice(capi, A, B, m, n, k, op, prec, stream):
    outs = []
    for _ in range(2):
        C = torch.full((m, n), float("nan"), device="cuda")
        d = capi.make_desc(m, n, k, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr(), op=op,
                           precision=prec)
        rc = capi.gemm_noalloc(d, stream)
        assert rc == capi.B2G_OK, capi.status_string(rc)
        torch.cuda.synchronize()
        assert not torch.isnan(C).any()
        outs.append(C)
    assert capi.noalloc_read_error(torch.cuda.current_device()) == 0
    return outs


# (m, n, k, op, precision): plain GEMMs with unaligned pitches (both operands
# staged), 3xTF32 (lo parts in the scratch even when aligned), triangular ops
# (their unit table is copied into the scratch, aligned or not; b2g_gemm keeps
# it in a per-device cache instead), up to a 12288 x 12288 triangle whose
# table holds thousands of units.
CASES = [(300, 250, 333, 0, 0), (129, 66, 1001, 0, 0),
         (300, 250, 333, 0, 1), (512, 384, 256, 0, 1),
         (300, 300, 300, 1, 0), (513, 513, 513, 2, 0), (1024, 1024, 1024, 1, 0),
         (12288, 12288, 12288, 1, 0)]


@pytest.mark.parametrize("m,n,k,op,prec", CASES)
def test_noalloc_matches_b2g_gemm_on_two_calls_in_a_row(capi, m, n, k, op, prec):
    stream = torch.cuda.current_stream().cuda_stream
    A, B = _inputs(m + 7 * n + 13 * k + op, m, n, k, op)
    C_ref, ws_bytes = _with_workspace(capi, A, B, m, n, k, op, prec, stream)
    d = capi.make_desc(m, n, k, a=A.data_ptr(), b=B.data_ptr(), c=C_ref.data_ptr(), op=op,
                       precision=prec)
    plan = capi.plan(d, torch.cuda.get_device_properties(0).multi_processor_count)
    assert plan.workspace_bytes == ws_bytes <= capi.NOALLOC_SCRATCH_BYTES
    if op == 0:        # staged operands or 3xTF32 lo parts: workspace for b2g_gemm
        assert ws_bytes > 0
    tol = O.TOL["tf32" if prec == 0 else "3xtf32"]
    C1, C2 = _noalloc_twice(capi, A, B, m, n, k, op, prec, stream)
    for C in (C1, C2):
        if m <= 2048:
            assert O.rel_fro(C.double().cpu().numpy(), C_ref.double().cpu().numpy()) <= tol
            assert O.rel_fro(C.double().cpu().numpy(), _oracle(A, B, op)) <= tol
        else:   # large triangular case: compare on the GPU
            rel = float(((C.double() - C_ref.double()).norm() / C_ref.double().norm()).item())
            assert rel <= tol
        if op:
            masked = torch.tril(C, -1) if op == 1 else torch.triu(C, 1)
            assert torch.count_nonzero(masked).item() == 0


def test_noalloc_rejects_staging_beyond_its_scratch(capi):
    # 4096 x 4095 needs a 64 MiB staged copy of A: more than the 16 MiB scratch.
    m, n, k = 4096, 64, 4095
    A = torch.zeros(m, k, device="cuda")
    B = torch.zeros(k, n, device="cuda")
    C = torch.zeros(m, n, device="cuda")
    d = capi.make_desc(m, n, k, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr())
    assert capi.lib().b2g_gemm_workspace_bytes(d) > capi.NOALLOC_SCRATCH_BYTES
    assert capi.gemm_noalloc(d) == capi.B2G_ERR_SCRATCH_LIMIT
    assert "scratch" in capi.status_string(capi.B2G_ERR_SCRATCH_LIMIT)


def test_noalloc_rejects_3xtf32_beyond_its_scratch(capi):
    # Aligned operands, but 3xTF32 keeps lo copies of A and B (2 x 16 MiB here).
    m = n = k = 2048
    A = torch.zeros(m, k, device="cuda")
    B = torch.zeros(k, n, device="cuda")
    C = torch.zeros(m, n, device="cuda")
    d = capi.make_desc(m, n, k, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr(),
                       precision=capi.PREC_3XTF32)
    assert capi.gemm_noalloc(d) == capi.B2G_ERR_SCRATCH_LIMIT
    d.precision = capi.PREC_TF32          # the same aligned call in TF32 needs no scratch
    assert capi.lib().b2g_gemm_workspace_bytes(d) == 0
    assert capi.gemm_noalloc(d) == capi.B2G_OK
    torch.cuda.synchronize()


CHILD = r"""
import importlib, json, sys, torch
sys.path.insert(0, sys.argv[1])
capi = importlib.import_module("cupilot-kernels_b200.capi")
g = torch.Generator().manual_seed(5)
m, n, k = 300, 250, 333
A = torch.randn(m, k, generator=g).cuda()
B = torch.randn(k, n, generator=g).cuda()
ref = (A.double() @ B.double())
res = {}
for i in range(2):
    C = torch.zeros(m, n, device="cuda")
    d = capi.make_desc(m, n, k, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr())
    res[f"rc{i}"] = capi.gemm_noalloc(d, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    res[f"code{i}"] = capi.noalloc_read_error(0)
    res[f"err{i}"] = float(((C.double() - ref).norm() / ref.norm()).item())
print(json.dumps(res))
"""


def test_noalloc_bounded_wait_is_reported():
    """The first call withholds its accumulator-ready signal (test hook), the
    epilogue's bounded wait gives up and records 0x105 in this path's own
    error word; b2g_noalloc_read_error returns it, and the next call in the
    same context is correct and reports 0."""
    env = dict(os.environ, B2G_TEST_STALL_ONCE="1", B2G_WAIT_LIMIT_MS="50")
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["rc0"] == 0 and out["code0"] == 0x105, out
    assert out["rc1"] == 0 and out["code1"] == 0 and out["err1"] <= 1e-2, out
