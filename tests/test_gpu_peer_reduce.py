"""The cross-GPU K-split sum (b2g_splitk_peer_reduce) on the GPU.

* One GPU, protocol only: two mailboxes on one device stand for rank 0
  (root) and rank 1.  The device is synchronised after each emulated
  rank's call (rank 1's push, then the root's reduce), so no kernel ever
  waits for another kernel running beside it: the flags a kernel waits on
  were set by a kernel that had finished before it was launched.  Several
  epochs run one after another (the landing slots alternate, the credits
  advance), and the sum is checked bit for bit (out = P0 + P1 in fp32) and
  against the fp64 oracle.
* One GPU, bounded wait: the root reduces an epoch nobody pushed (a flag
  that nothing sets); with B2G_WAIT_LIMIT_MS=50 the wait gives up, the
  kernel records 0x202 in the device error word and returns, and the next
  GEMM in the same context is correct.
* Two GPUs (skipped with fewer): torchrun with two ranks runs the large-K
  product split over K through Partitioner.split_k_matmul(method="peer"),
  three calls in a row, three through the fused kernel (method="fused",
  b2g_gemm_splitk_peer), then three pipelined calls (split_k_matmul_async:
  the sums on a side stream behind the GEMMs) and a join, each result
  checked on the root against a float64 product.
* One GPU, fused kernel: b2g_gemm_splitk_peer with two emulated ranks run
  one after the other (rank 1 first), epochs alternating with the
  stand-alone path on the same mailboxes; and its bounded wait as the root
  of an epoch nobody pushed.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import REPO, import_pkg
from oracle import gemm_oracle as O

pytestmark = pytest.mark.gpu


def test_peer_reduce_protocol_on_one_gpu(capi, ops):
    m = n = 256
    elems = m * n
    mb = [capi.peer_mailbox_create(elems, 2)[0] for _ in range(2)]
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(1)
    try:
        for epoch in range(1, 6):
            k = 4096 * epoch
            A = torch.randn(m, k, generator=g, device="cuda")
            B = torch.randn(k, n, generator=g, device="cuda")
            h = k // 2
            P1 = ops.p2.forward(A[:, h:].contiguous(), B[h:].contiguous())
            rc = capi.splitk_peer_reduce(P1.data_ptr(), 0, elems, mb, 1, 0, epoch, stream)
            assert rc == capi.B2G_OK, capi.status_string(rc)
            torch.cuda.synchronize()          # rank 1's push has finished
            out = ops.p2.forward(A[:, :h].contiguous(), B[:h].contiguous())
            P0 = out.clone()
            rc = capi.splitk_peer_reduce(0, out.data_ptr(), elems, mb, 0, 0, epoch, stream)
            assert rc == capi.B2G_OK, capi.status_string(rc)
            torch.cuda.synchronize()
            assert torch.equal(out, P0 + P1)
            err = O.rel_fro(out.double().cpu().numpy(), O.large_k(A.cpu().numpy(), B.cpu().numpy()))
            assert err <= O.TOL["tf32"]
        assert ops.read_device_error(torch.cuda.current_device()) == 0
    finally:
        for p in mb:
            capi.peer_mailbox_destroy(p)


@pytest.mark.parametrize("k", [256, 65536])
def test_fused_splitk_peer_on_one_gpu(capi, ops, k):
    """b2g_gemm_splitk_peer (product and cross-GPU sum in one kernel) with
    two emulated ranks on one device, rank 1 first, the device synchronised
    between the calls; epochs alternate between the fused path and the
    stand-alone GEMM + b2g_splitk_peer_reduce on the same mailboxes.  At
    k = 256 no launch splits K, so every partial is deterministic and the
    root's sum must equal P0 + P1 bit for bit; at k = 65536 (split-K inside
    each rank) the sum is checked against the fp64 oracle."""
    m = n = 256
    elems = m * n
    mb = [capi.peer_mailbox_create(elems, 2)[0] for _ in range(2)]
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(5)
    native = import_pkg().native()
    try:
        for epoch in range(1, 7):
            A = torch.randn(m, k, generator=g, device="cuda")
            B = torch.randn(k, n, generator=g, device="cuda")
            h = k // 2
            A1, B1 = A[:, h:].contiguous(), B[h:].contiguous()
            A0, B0 = A[:, :h].contiguous(), B[:h].contiguous()
            fused = epoch % 2 == 1
            if fused:
                C1 = native.splitk_peer_matmul(A1, B1, mb, 1, 0, epoch)
                torch.cuda.synchronize()      # rank 1's kernel has finished
                P1 = C1.clone()
                out = native.splitk_peer_matmul(A0, B0, mb, 0, 0, epoch)
                torch.cuda.synchronize()
            else:
                P1 = ops.p2.forward(A1, B1)
                rc = capi.splitk_peer_reduce(P1.data_ptr(), 0, elems, mb, 1, 0, epoch, stream)
                assert rc == capi.B2G_OK, capi.status_string(rc)
                torch.cuda.synchronize()
                out = ops.p2.forward(A0, B0)
                rc = capi.splitk_peer_reduce(0, out.data_ptr(), elems, mb, 0, 0, epoch, stream)
                assert rc == capi.B2G_OK, capi.status_string(rc)
                torch.cuda.synchronize()
            if k == 256:
                P0 = ops.p2.forward(A0, B0)
                assert torch.equal(out, P0 + P1), epoch
            err = O.rel_fro(out.double().cpu().numpy(), O.large_k(A.cpu().numpy(), B.cpu().numpy()))
            assert err <= O.TOL["tf32"], (epoch, err)
        assert ops.read_device_error(torch.cuda.current_device()) == 0
    finally:
        for p in mb:
            capi.peer_mailbox_destroy(p)


TIMEOUT_CHILD = r"""
import importlib, json, sys, time, torch
sys.path.insert(0, sys.argv[1])
ops = importlib.import_module("cupilot-kernels_b200.ops")
capi = importlib.import_module("cupilot-kernels_b200.capi")
elems = 64 * 64
mb = [capi.peer_mailbox_create(elems, 2)[0] for _ in range(2)]
out = torch.zeros(elems, device="cuda")
t0 = time.time()
rc = capi.splitk_peer_reduce(0, out.data_ptr(), elems, mb, 0, 0, 1,
                             torch.cuda.current_stream().cuda_stream)
torch.cuda.synchronize()
waited = time.time() - t0
code = ops.read_device_error(0)
A = torch.randn(300, 200, device="cuda"); B = torch.randn(200, 100, device="cuda")
C = ops.p2.forward(A, B)
ref = A.double() @ B.double()
err = float(((C.double() - ref).norm() / ref.norm()).item())
for p in mb:
    capi.peer_mailbox_destroy(p)
print(json.dumps({"rc": rc, "code": code, "waited": waited, "err_after": err,
                  "out_untouched": bool((out == 0).all().item()),
                  "code_after": ops.read_device_error(0)}))
"""


FUSED_TIMEOUT_CHILD = r"""
import importlib, json, sys, time, torch
sys.path.insert(0, sys.argv[1])
ops = importlib.import_module("cupilot-kernels_b200.ops")
capi = importlib.import_module("cupilot-kernels_b200.capi")
native = importlib.import_module("cupilot-kernels_b200").native()
m = n = 128
mb = [capi.peer_mailbox_create(m * n, 2)[0] for _ in range(2)]
A = torch.randn(m, 512, device="cuda"); B = torch.randn(512, n, device="cuda")
t0 = time.time()
C = native.splitk_peer_matmul(A, B, mb, 0, 0, 1)     # root of an epoch nobody pushed
torch.cuda.synchronize()
waited = time.time() - t0
code = ops.read_device_error(0)
ref = A.double() @ B.double()
own = float(((C.double() - ref).norm() / ref.norm()).item())   # only its own partial
A2 = torch.randn(300, 200, device="cuda"); B2 = torch.randn(200, 100, device="cuda")
C2 = ops.p2.forward(A2, B2)
ref2 = A2.double() @ B2.double()
err = float(((C2.double() - ref2).norm() / ref2.norm()).item())
for p in mb:
    capi.peer_mailbox_destroy(p)
print(json.dumps({"code": code, "waited": waited, "own": own, "err_after": err,
                  "code_after": ops.read_device_error(0)}))
"""


def test_fused_splitk_bounded_wait_reports_and_context_survives():
    """The fused kernel as root of an epoch no rank pushed: its wait for the
    ready flags gives up after B2G_WAIT_LIMIT_MS, records 0x202 and the
    kernel ends with the root's own partial in C; the next GEMM is correct."""
    env = dict(os.environ, B2G_WAIT_LIMIT_MS="50")
    r = subprocess.run([sys.executable, "-c", FUSED_TIMEOUT_CHILD, str(REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["code"] == 0x202 and out["waited"] < 30, out
    assert out["own"] <= 1e-2, out
    assert out["err_after"] <= 1e-2 and out["code_after"] == 0, out


def test_peer_reduce_bounded_wait_reports_and_context_survives():
    env = dict(os.environ, B2G_WAIT_LIMIT_MS="50")
    r = subprocess.run([sys.executable, "-c", TIMEOUT_CHILD, str(REPO)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["rc"] == 0 and out["code"] == 0x202, out
    assert out["waited"] < 30 and out["out_untouched"], out
    assert out["err_after"] <= 1e-2 and out["code_after"] == 0, out


MULTI = r"""
import importlib, json, os, sys, torch
import torch.distributed as dist
sys.path.insert(0, sys.argv[1])
part_mod = importlib.import_module("cupilot-kernels_b200.partition")
ops = importlib.import_module("cupilot-kernels_b200.ops")
p = part_mod.init_node("nccl", timeout_s=60)
m = n = 256
k = 65536
res = []
for step in range(3):
    g = torch.Generator(device="cuda").manual_seed(100 + step)
    A = torch.randn(m, k, generator=g, device="cuda")       # same on every rank
    B = torch.randn(k, n, generator=g, device="cuda")
    k0, k1 = p.k_range(k)
    C = p.split_k_matmul(A[:, k0:k1].contiguous(), B[k0:k1].contiguous(), root=0, method="peer")
    torch.cuda.synchronize()
    if p.rank == 0:
        ref = A.double() @ B.double()
        res.append(float(((C.double() - ref).norm() / ref.norm()).item()))
    else:
        assert C is None
# Fused: product and cross-GPU sum in one kernel per step.
for step in range(3):
    g = torch.Generator(device="cuda").manual_seed(300 + step)
    A = torch.randn(m, k, generator=g, device="cuda")
    B = torch.randn(k, n, generator=g, device="cuda")
    k0, k1 = p.k_range(k)
    C = p.split_k_matmul(A[:, k0:k1].contiguous(), B[k0:k1].contiguous(), root=0, method="fused")
    torch.cuda.synchronize()
    if p.rank == 0:
        ref = A.double() @ B.double()
        res.append(float(((C.double() - ref).norm() / ref.norm()).item()))
    else:
        assert C is None
# Pipelined: three sums on the side stream behind three GEMMs, then join.
outs, refs = [], []
for step in range(3):
    g = torch.Generator(device="cuda").manual_seed(200 + step)
    A = torch.randn(m, k, generator=g, device="cuda")
    B = torch.randn(k, n, generator=g, device="cuda")
    k0, k1 = p.k_range(k)
    outs.append(p.split_k_matmul_async(A[:, k0:k1].contiguous(), B[k0:k1].contiguous(), root=0))
    refs.append((A, B))
p.join()
torch.cuda.synchronize()
if p.rank == 0:
    for C, (A, B) in zip(outs, refs):
        ref = A.double() @ B.double()
        res.append(float(((C.double() - ref).norm() / ref.norm()).item()))
err_code = ops.read_device_error(torch.cuda.current_device())
codes = [None] * p.world
dist.all_gather_object(codes, err_code)
if p.rank == 0:
    print(json.dumps({"errs": res, "codes": codes}))
dist.barrier()
dist.destroy_process_group()
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_reduce_two_gpus(tmp_path):
    script = tmp_path / "multi.py"
    script.write_text(MULTI)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
                        str(script), str(REPO)], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    out = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][-1])
    assert out["codes"] == [0, 0], out
    assert len(out["errs"]) == 9 and max(out["errs"]) <= 1e-2, out
