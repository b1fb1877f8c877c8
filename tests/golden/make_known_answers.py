"""Generate tests/golden/known_answers.json from closed-form formulas.

Each case gives small integer-valued inputs and the exact expected output,
written down from the mathematics of the operator (not computed by the
oracle), so the oracle can be pinned against them.  Run from the repo root:
    python tests/golden/make_known_answers.py
"""
import json
from pathlib import Path


def ones_triu(n):
    return [[1.0 if j >= i else 0.0 for j in range(n)] for i in range(n)]


def ones_tril(n):
    return [[1.0 if j <= i else 0.0 for j in range(n)] for i in range(n)]


def full(n, v):
    return [[v] * n for _ in range(n)]


cases = []
n = 7
# triu(1)·triu(1): entry (i, j) counts k with i <= k <= j -> j - i + 1 above the diagonal.
cases.append({"pid": 14, "name": "upper_ones", "A": ones_triu(n), "B": ones_triu(n),
              "C": [[float(j - i + 1) if j >= i else 0.0 for j in range(n)] for i in range(n)]})
# Full ones in, upper-triangular semantics mask the inputs first: same answer.
cases.append({"pid": 14, "name": "upper_masks_inputs", "A": full(n, 1.0), "B": full(n, 1.0),
              "C": [[float(j - i + 1) if j >= i else 0.0 for j in range(n)] for i in range(n)]})
cases.append({"pid": 15, "name": "lower_ones", "A": ones_tril(n), "B": ones_tril(n),
              "C": [[float(i - j + 1) if j <= i else 0.0 for j in range(n)] for i in range(n)]})
cases.append({"pid": 15, "name": "lower_masks_inputs", "A": full(n, 1.0), "B": full(n, 1.0),
              "C": [[float(i - j + 1) if j <= i else 0.0 for j in range(n)] for i in range(n)]})
# [[1,2],[3,4]] . [[5,6],[7,8]] = [[19,22],[43,50]]
cases.append({"pid": 1, "name": "square_2x2", "A": [[1.0, 2.0], [3.0, 4.0]],
              "B": [[5.0, 6.0], [7.0, 8.0]], "C": [[19.0, 22.0], [43.0, 50.0]]})
# A stored (K=2, M=3): A^T B with B (2, 2).  A^T = [[1,4],[2,5],[3,6]].
cases.append({"pid": 16, "name": "at_b", "A": [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]],
              "B": [[1.0, 0.0], [0.0, 1.0]], "C": [[1.0, 4.0], [2.0, 5.0], [3.0, 6.0]]})
# A (2,3) . B^T with B stored (N=2, K=3): rows dot rows.
cases.append({"pid": 17, "name": "a_bt", "A": [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]],
              "B": [[1.0, 1.0, 1.0], [1.0, 0.0, -1.0]], "C": [[6.0, -2.0], [15.0, -2.0]]})
# A^T B^T: A stored (K=2, M=2), B stored (N=2, K=2): [[1,3],[2,4]] . [[0,1],[1,0]].
cases.append({"pid": 18, "name": "at_bt", "A": [[1.0, 2.0], [3.0, 4.0]],
              "B": [[0.0, 1.0], [1.0, 0.0]], "C": [[3.0, 1.0], [4.0, 2.0]]})
# diag(a) B scales rows.
cases.append({"pid": 12, "name": "diag", "A": [2.0, -1.0, 0.5], "B": [[1.0, 2.0], [3.0, 4.0],
              [8.0, 6.0]], "C": [[2.0, 4.0], [-3.0, -4.0], [4.0, 3.0]]})
# Batched: two independent 2x2 products.
cases.append({"pid": 3, "name": "bmm", "A": [[[1.0, 0.0], [0.0, 1.0]], [[2.0, 0.0], [0.0, 2.0]]],
              "B": [[[1.0, 2.0], [3.0, 4.0]], [[1.0, 1.0], [1.0, 1.0]]],
              "C": [[[1.0, 2.0], [3.0, 4.0]], [[2.0, 2.0], [2.0, 2.0]]]})
# 4-D einsum with all-ones operands: every output equals l.
b, i, j, l, k = 2, 2, 3, 5, 4
cases.append({"pid": 11, "name": "einsum_ones",
              "A": [[[[1.0] * l for _ in range(j)] for _ in range(i)] for _ in range(b)],
              "B": [[1.0] * k for _ in range(l)],
              "C": [[[[float(l)] * k for _ in range(j)] for _ in range(i)] for _ in range(b)]})
# 3-D tensor x matrix.
cases.append({"pid": 10, "name": "tensor3d", "A": [[[1.0, 2.0]], [[3.0, 4.0]]],
              "B": [[1.0, 0.0, 1.0], [0.0, 1.0, 1.0]],
              "C": [[[1.0, 2.0, 3.0]], [[3.0, 4.0, 7.0]]]})

# GEMV: [[1,2,3],[4,5,6]] . [1,0,-1]^T = [-2, -2]
cases.append({"pid": 4, "name": "gemv", "A": [[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]],
              "B": [[1.0], [0.0], [-1.0]], "C": [[-2.0], [-2.0]]})
# Matrix x scalar.
cases.append({"pid": 5, "name": "scalar", "A": [[1.0, -2.0], [0.5, 3.0]], "B": 4.0,
              "C": [[4.0, -8.0], [2.0, 12.0]]})

# Pointwise conv, input (1, 2, 2, 2): channel 0 = [[1,2],[3,4]], channel 1 = [[5,6],[7,8]];
# weight (3, 2, 1, 1) rows [1,0], [0,1], [1,-1]; bias [0.5, -1, 2]:
# out channel 0 = x0 + 0.5, channel 1 = x1 - 1, channel 2 = x0 - x1 + 2 = -2 everywhere.
x0, x1 = [[1.0, 2.0], [3.0, 4.0]], [[5.0, 6.0], [7.0, 8.0]]
wt = [[[[1.0]], [[0.0]]], [[[0.0]], [[1.0]]], [[[1.0]], [[-1.0]]]]
cases.append({"pid": 87, "name": "conv1x1_bias", "A": [[x0, x1]], "B": wt, "bias": [0.5, -1.0, 2.0],
              "C": [[[[1.5, 2.5], [3.5, 4.5]], [[4.0, 5.0], [6.0, 7.0]],
                     [[-2.0, -2.0], [-2.0, -2.0]]]]})
cases.append({"pid": 87, "name": "conv1x1_nobias", "A": [[x0, x1]], "B": wt,
              "C": [[x0, x1, [[-4.0, -4.0], [-4.0, -4.0]]]]})

# Attention: identical keys give a uniform softmax, so every output row is the
# mean of V's rows; a single key gives V itself.
cases.append({"pid": 97, "name": "sdpa_uniform", "A": [[[[1.0, 0.0], [0.0, 1.0]]]],
              "B": [[[[1.0, 1.0], [1.0, 1.0]]]], "V": [[[[1.0, 2.0], [3.0, 4.0]]]],
              "C": [[[[2.0, 3.0], [2.0, 3.0]]]]})
cases.append({"pid": 97, "name": "sdpa_one_key", "A": [[[[0.5, -2.0]]]], "B": [[[[3.0, 1.0]]]],
              "V": [[[[-1.0, 7.0]]]], "C": [[[[-1.0, 7.0]]]]})

out = Path(__file__).with_name("known_answers.json")
out.write_text(json.dumps({"cases": cases}, indent=0))
print(f"wrote {len(cases)} cases to {out}")
