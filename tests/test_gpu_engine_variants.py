"""Every engine variant (tile shape x CTA pairing) against the fp64 oracle.

The dispatcher normally picks one tile shape per problem; B2G_TILE pins it.
It is read once per process, so each variant runs in a child process.
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
from oracle import gemm_oracle as O
out = []
for (m, n, k, ta, tb, mode) in json.loads(sys.argv[2]):
    g = torch.Generator().manual_seed(m * 31 + n * 7 + k)
    A = torch.randn(*((k, m) if ta else (m, k)), generator=g)
    B = torch.randn(*((n, k) if tb else (k, n)), generator=g)
    with ops.precision(mode):
        C = ops.gemm(A.cuda(), B.cuda(), bool(ta), bool(tb), 0)
    Aop = A.numpy().T if ta else A.numpy()
    Bop = B.numpy().T if tb else B.numpy()
    out.append(O.rel_fro(C.cpu().double().numpy(), O.matmul(Aop, Bop)))
assert ops.read_device_error(0) == 0
print(json.dumps(out))
"""

SHAPES = [(1, 1, 1, 0, 0, "tf32"), (300, 700, 200, 0, 0, "tf32"), (512, 1536, 256, 1, 1, "tf32"),
          (256, 1024, 96, 0, 1, "tf32"), (130, 600, 1000, 1, 0, "tf32"),
          (1024, 1024, 4096, 0, 0, "tf32"), (96, 512, 64, 0, 0, "3xtf32")]


@pytest.mark.parametrize("tile", ["pair512", "pair256", "pair128", "single256", "single128"])
def test_variant_matches_oracle(tile):
    env = dict(os.environ, B2G_TILE=tile)
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO), json.dumps(SHAPES)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    errs = json.loads(r.stdout.strip().splitlines()[-1])
    for shape, e in zip(SHAPES, errs):
        tol = 1e-3 if shape[-1] == "3xtf32" else 1e-2
        assert e <= tol, (tile, shape, e)
