"""The dynamic unit schedule far past its ring's wrap, at small sizes.

Plain GEMMs with more work units than CTAs (pairs) draw their units from a
global counter; the pair leader publishes each drawn index into a 32-slot
ring in shared memory that every role reads, the slot's mbarrier phase
flipping on each pass (gemm_engine.cuh, UnitSource::get).  On 148 SMs only
configs with thousands of units pass the ring more than once per CTA.
B2G_MAX_SMS=8 plans every launch as if the GPU had 8 SMs, so a persistent
grid of 8 CTAs (4 pairs) walks 64-1024 units each here, wrapping the ring
2-32 times, for every tile shape the dispatcher can pick (B2G_TILE), in
both precision modes, batched and with split K.  Each child process checks
its outputs against a float64 product and the device error word.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

CHILD = r"""
import importlib, json, sys, torch
sys.path.insert(0, sys.argv[1])
ops = importlib.import_module("cupilot-kernels_b200.ops")
capi = importlib.import_module("cupilot-kernels_b200.capi")
out = []
g = torch.Generator(device="cuda").manual_seed(11)
cases = [("nn", 1, 4096, 4096, 64), ("nn", 1, 2048, 2048, 512), ("nn", 1, 1000, 1500, 300),
         ("bmm", 24, 256, 512, 256), ("splitk", 1, 256, 256, 65536)]
for kind, batch, m, n, k in cases:
    A = torch.randn(batch, m, k, generator=g, device="cuda")
    B = torch.randn(batch, k, n, generator=g, device="cuda")
    for mode in ("tf32", "3xtf32"):
        with ops.precision(mode):
            C = ops.p3.forward(A, B) if batch > 1 else ops.p2.forward(A[0], B[0])[None]
        torch.cuda.synchronize()
        ref = torch.matmul(A.double(), B.double())
        err = float(((C.double() - ref).norm() / ref.norm()).item())
        d = capi.make_desc(m, n, k, batch=batch, a=A.data_ptr(), b=B.data_ptr(), c=C.data_ptr(),
                           stride_a=m * k, stride_b=k * n, stride_c=m * n,
                           precision=0 if mode == "tf32" else 1)
        p = capi.plan(d, 8)
        slots = p.grid // p.cluster_ctas
        out.append({"case": [kind, batch, m, n, k], "mode": mode, "err": err,
                    "units": p.work_units, "slots": slots, "block_n": p.block_n,
                    "ctas": p.cluster_ctas, "splits": p.splits})
print(json.dumps({"cases": out, "device_error": ops.read_device_error(0)}))
"""

TILES = ["pair256", "pair512", "pair128", "single256", "single128"]


@pytest.mark.parametrize("tile", TILES)
def test_dynamic_unit_ring_wraps(tile):
    env = dict(os.environ, B2G_MAX_SMS="8", B2G_TILE=tile)
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["device_error"] == 0, res
    wraps = 0
    for c in res["cases"]:
        tol = 1e-2 if c["mode"] == "tf32" else 1e-3
        assert c["err"] <= tol, c
        assert c["slots"] <= 8, c
        wraps = max(wraps, c["units"] // max(c["slots"], 1) // 32)
    assert wraps >= 2, res        # the ring went round at least twice in some CTA
