"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait in the GEMM engine is bounded.  B2G_TEST_STALL_ONCE=1
makes the first GEMM of a process withhold its "accumulator ready" signal
(a flag that nothing sets), B2G_WAIT_LIMIT_MS=50 shortens the bound; the
epilogue's wait then runs out, the kernel writes an error code into the
device error word, every role unwinds (draining its own loads and MMAs) and
the kernel returns.  The host reads the code, and the context stays usable:
the next GEMM in the same process is correct.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

CHILD = r"""
import importlib, json, sys, time, torch
sys.path.insert(0, sys.argv[1])
ops = importlib.import_module("cupilot-kernels_b200.ops")
from oracle import gemm_oracle as O
g = torch.Generator().manual_seed(3)
A = torch.randn(512, 384, generator=g)
B = torch.randn(384, 640, generator=g)
t0 = time.time()
C1 = ops.p2.forward(A.cuda(), B.cuda())        # stalls by design, then unwinds
torch.cuda.synchronize()
stalled_s = time.time() - t0
code = ops.read_device_error(0)
C2 = ops.p2.forward(A.cuda(), B.cuda())        # normal launch in the same context
torch.cuda.synchronize()
err = O.rel_fro(C2.cpu().double().numpy(), O.standard(A.numpy(), B.numpy()))
print(json.dumps({"code": code, "stalled_s": stalled_s, "err_after": err,
                  "code_after": ops.read_device_error(0)}))
"""


def test_bounded_wait_reports_and_context_survives():
    env = dict(os.environ, B2G_TEST_STALL_ONCE="1", B2G_WAIT_LIMIT_MS="50")
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["code"] == 0x105, out           # kErrWaitTmemFull: the epilogue gave up
    assert out["stalled_s"] < 30, out
    assert out["err_after"] <= 1e-2, out
    assert out["code_after"] == 0, out
