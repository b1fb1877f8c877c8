"""The CPU oracle against the closed-form known answers (no GPU)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import gemm_oracle as O

GOLDEN = Path(__file__).parent / "golden" / "known_answers.json"


def _cases():
    return json.loads(GOLDEN.read_text())["cases"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: f"p{c['pid']}-{c['name']}")
def test_known_answers(case):
    f = O.BY_PID[case["pid"]]
    B = case["B"] if case["pid"] == 5 else np.array(case["B"], dtype=np.float32)
    extra = [np.array(case[key], dtype=np.float32) for key in ("bias", "V") if key in case]
    got = f(np.array(case["A"], dtype=np.float32), B, *extra)
    np.testing.assert_array_equal(np.asarray(got, dtype=np.float64), np.array(case["C"]))


def test_every_operator_is_pinned_or_shares_a_pinned_formula():
    pinned = {c["pid"] for c in _cases()}
    # Plain C = A B operators share one formula with the pinned square case.
    plain = {1, 2, 6, 7, 8, 9, 13}
    assert set(O.BY_PID) <= pinned | plain


def test_rel_fro_properties():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 7))
    assert O.rel_fro(x, x) == 0.0
    assert abs(O.rel_fro(1.01 * x, x) - 0.01) < 1e-12
    assert O.rel_fro(np.zeros(3), np.zeros(3)) == 0.0


def test_triangular_semantics_mask_inputs():
    rng = np.random.default_rng(1)
    A = rng.standard_normal((9, 9))
    B = rng.standard_normal((9, 9))
    up = O.upper_tri(A, B)
    assert np.all(np.tril(up, -1) == 0)
    np.testing.assert_allclose(up, np.triu(np.triu(A) @ np.triu(B)))
    lo = O.lower_tri(A, B)
    assert np.all(np.triu(lo, 1) == 0)


def test_diag_single_rounding():
    a = np.float32([3.0, 1.0 / 3.0])
    B = np.float32([[1.0 / 3.0, 7.0], [3.0, 0.1]])
    out = O.diag(a, B)
    assert out.dtype == np.float32
    assert out[0, 0] == np.float32(np.float32(3.0) * np.float32(1.0 / 3.0))
