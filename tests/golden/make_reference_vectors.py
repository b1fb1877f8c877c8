"""Generate tests/golden/reference_outputs.npz from the reference's own kernels.

Runs on a GPU box where oracle/build_ref.py has compiled the reference
kernels (kernels/<PID>_*.cu, unmodified, sm_100a).  For each operator it
draws small seeded N(0,1) inputs on the CPU (torch.Generator, so the test
can regenerate them bit-for-bit), runs the reference's Part-3 function and
stores its output (row subsets for the larger ones).  Shapes stay inside
each reference kernel's own contract (tile multiples, K7's K = 64, K9's
inner dimension <= 32, K87's channel and tile multiples, K16's block swizzle needing M and N multiples of 512,
kernels/16_Matmul_with_transposed_A_best_kernel.cu:18-40).  K2 runs at its
own hard-coded 2048 x 8192 x 4096 (kernels/2_Standard_matrix_multiplication_best_kernel.cu:16-18)
and keeps a 16 x 512 corner of its output.  K4 runs only where its loop
bound cannot wrap: `num_vectors - blockDim.x*3` (kernels/4_Matrix_vector_multiplication_best_kernel.cu:22)
mixes int with unsigned, so below 3072 float4s per row (K < 12288 at its
1024 threads) the bound becomes a huge unsigned value and the loop reads
past the row (its first call here, at K = 1024, raised an illegal memory
access); K = 16384 is inside its contract.  Case 114 is K14 on UNMASKED
inputs: K14 masks its own operands (kernels/14_...:74-75,84-85), which
the oracle's triu(triu(A) triu(B)) must reproduce.

    python tests/golden/make_reference_vectors.py [pid,pid,...]

With a list of problem IDs only those cases are (re)generated and merged
into the existing fixture.
"""
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

# case -> (list of input shapes, part of the output to keep: leading rows, or
# a (rows, cols) corner); at most 64 rows are stored to keep the fixture small.
SCALE = 2.5   # the scalar operand of K5
CASES = {
    2: ([(2048, 8192), (8192, 4096)], (16, 512)),   # K2's hard-coded shape; corner kept
    4: ([(64, 16384), (16384, 1)], 64),
    114: ([(256, 256), (256, 256)], 64),            # K14 on unmasked inputs
    5: ([(64, 256)], 64),
    1: ([(256, 256), (256, 256)], 64),
    3: ([(2, 256, 64), (2, 64, 256)], 64),
    6: ([(64, 2048), (2048, 64)], 64),
    7: ([(256, 64), (64, 256)], 64),
    8: ([(67, 33), (33, 45)], 64),
    9: ([(1024, 32), (32, 1024)], 64),
    10: ([(2, 128, 64), (64, 128)], 64),
    11: ([(1, 2, 32, 64), (64, 256)], 64),
    12: ([(64,), (64, 96)], 64),
    13: ([(256, 256), (256, 256)], 64),
    14: ([(256, 256), (256, 256)], 64),
    15: ([(256, 256), (256, 256)], 64),
    16: ([(64, 512), (64, 512)], 64),     # K16's 8x8 block swizzle needs M, N % 512
    17: ([(128, 64), (96, 64)], 64),
    18: ([(64, 64), (256, 64)], 64),
    # K87: input (N, Cin, H, W), weight (Cout, Cin, 1, 1), bias (Cout,).  Its
    # contract (kernels/87_conv_pointwise_2D_best_kernel.cu:183-330): unguarded
    # 8-wide weight loads need Cout % 128 == 0 and Cin % 8 == 0, 8-wide input
    # loads need H*W % 8 == 0, and full 64-position tiles N*H*W % 64 == 0.
    87: ([(2, 40, 4, 16), (128, 40, 1, 1), (128,)], None),
    # K97: fp16 Q, K, V (batch, heads, seq, dim); its loops assume seq == 512
    # and dim == 1024 (kernels/97_ScaledDotProductAttention_best_kernel.cu:9-10,
    # :102, :182).  First 16 query rows kept.
    97: ([(1, 1, 512, 1024)] * 3, 16),
}
SEED0 = 1234
# Case -> the reference kernel (problem ID) it runs.
KERNEL = {114: 14}


def inputs(pid):
    g = torch.Generator().manual_seed(SEED0 + pid)
    shapes, _ = CASES[pid]
    ts = [torch.randn(*s, generator=g) for s in shapes]
    if pid == 5:
        ts.append(SCALE)
    if pid == 13:
        ts = [(t + t.T) / 2 for t in ts]
    if pid == 14:
        ts = [torch.triu(t) for t in ts]
    if pid == 15:
        ts = [torch.tril(t) for t in ts]
    if pid == 97:
        ts = [t.half() for t in ts]
    return ts


def keep_part(C, keep):
    """The stored part of an output: leading rows (int) or a leading
    (rows, cols) corner of every output matrix."""
    if keep is None:
        return C
    if isinstance(keep, tuple):
        return C[..., : keep[0], : keep[1]]
    return C[..., :keep, :]


def main():
    from oracle import build_ref

    path = Path(__file__).with_name("reference_outputs.npz")
    only = {int(x) for x in sys.argv[1].split(",")} if len(sys.argv) > 1 else None
    out = dict(np.load(path)) if (only and path.exists()) else {}
    for pid, (_, keep) in CASES.items():
        if only and pid not in only:
            continue
        f = build_ref.load(KERNEL.get(pid, pid))
        A, B, *rest = inputs(pid)
        C = f(A.cuda(), B if pid == 5 else B.cuda(), *[t.cuda() for t in rest])
        torch.cuda.synchronize()
        C = keep_part(C.cpu().numpy(), keep)
        out[f"p{pid}"] = C.astype(np.float32)   # (fp16 outputs are exact in fp32)
        print(pid, C.shape, flush=True)
    np.savez_compressed(path, **out)


if __name__ == "__main__":
    main()
