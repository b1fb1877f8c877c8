"""The module-style boundary: ModelRef formulas against the oracle (CPU), and
ModelNew against ModelRef on every operator (GPU)."""
import numpy as np
import pytest
import torch

from conftest import import_pkg
from oracle import gemm_oracle as O


def _h():
    return import_pkg("harness")


@pytest.mark.parametrize("pid", [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 18, 87, 97])
def test_model_ref_matches_oracle(pid):
    h = _h()
    assert pid in h.pids()
    args = h.inputs(pid, small=True, device="cpu")
    if pid == 97:
        args = tuple(a[:, :, :64] for a in args)     # keep the CPU check quick
    got = h.model_ref(pid)(*args)
    want = O.BY_PID[pid](*[a.numpy() if torch.is_tensor(a) else a for a in args])
    err = O.rel_fro(np.asarray(got.double()), np.asarray(want))
    assert err <= (1e-3 if pid == 97 else 1e-5), err


@pytest.mark.gpu
@pytest.mark.parametrize("pid", [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 18, 87, 97])
def test_model_new_matches_model_ref(pid):
    h = _h()
    ok, err = h.check(pid, *h.inputs(pid, small=True))
    assert ok, f"pid {pid}: rel err {err:.3e}"
    assert isinstance(h.model_new(pid), torch.nn.Module)
