"""The C-ABI library on the host: loads, exports every declared symbol, and
its dispatcher plans correctly (pure host arithmetic, no GPU)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from conftest import REPO, import_pkg

HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_symbols():
    names = []
    for h in HEADERS:
        names += re.findall(r"^B2G_API\s+[\w\s\*]+?\b(b2g_\w+)\s*\(", h.read_text(), re.M)
    return names


def test_library_loads_and_exports_every_declared_symbol(capi):
    lib = capi.lib()
    names = declared_symbols()
    assert len(names) >= 7
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (b2g_\w+)", out))
    assert set(names) <= exported


def test_version_and_status_strings(capi):
    assert capi.lib().b2g_version() >= 100
    assert capi.status_string(0) == "ok"
    assert "workspace" in capi.status_string(capi.B2G_ERR_WORKSPACE)


def test_struct_layout_matches_header(capi):
    # 2 x int32 + 4 x int64 + 3 x (ptr, int64, int64, int32->padded) ... checked by size.
    assert ctypes.sizeof(capi.GemmDesc) == 8 + 32 + 3 * 32 - 8 + 16
    assert ctypes.sizeof(capi.GemmPlan) == 17 * 4 + 4 + 16


ALIGNED = 1 << 20   # a fake 16-byte-aligned device address: planning never dereferences


def _plan(capi, m, n, k, **kw):
    kw.setdefault("a", ALIGNED)
    kw.setdefault("b", ALIGNED)
    kw.setdefault("c", ALIGNED)
    return capi.plan(capi.make_desc(m, n, k, **kw))


def test_plan_square_2048(capi):
    p = _plan(capi, 2048, 2048, 2048)
    # CTA pairs on 256 x 256 units: 64 units on 128 SMs, one wave.
    assert (p.block_m, p.block_n, p.block_k) == (256, 256, 32)
    assert p.cluster_ctas == 2 and p.stages == 6
    assert p.splits == 1 and p.tiles_m == 8 and p.tiles_n == 8
    assert p.grid == 128 and p.work_units == 64
    assert p.a_mn_major == 0 and p.b_mn_major == 1
    assert p.stage_a == 0 and p.stage_b == 0 and p.workspace_bytes == 0
    assert p.tma_store == 1


def test_plan_transposes_set_majorness(capi):
    p = _plan(capi, 1024, 2048, 4096, trans_a=1, trans_b=1)
    assert p.a_mn_major == 1 and p.b_mn_major == 0
    # 32 units of 256 x 256 fill 64 SMs: K is split in two to fill 128.
    assert p.cluster_ctas == 2 and p.block_n == 256 and p.splits == 2 and p.grid == 128


def test_plan_triangular_3xtf32_uses_the_transform_variant(capi):
    p = _plan(capi, 300, 300, 300, op=capi.OP_TRI_UPPER, precision=capi.PREC_3XTF32)
    assert p.cluster_ctas == 1 and p.block_n == 128 and p.tri_diag == 0 and p.x3_split == 0


def test_plan_grid_is_even_for_pairs(capi):
    for m, n, k in [(256, 256, 256), (4096, 4096, 64), (300, 5000, 100), (8205, 5921, 2949)]:
        p = _plan(capi, m, n, k, a=ALIGNED, b=ALIGNED)
        if p.cluster_ctas == 2:
            assert p.grid % 2 == 0 and p.grid <= 148


def test_plan_short_k_prefers_single_cta_units(capi):
    # Output-bound (K <= 64): single-CTA 128 x 256 units store faster than pairs.
    for m, n, k in [(16384, 16384, 32), (16384, 16384, 64)]:
        p = _plan(capi, m, n, k)
        assert p.cluster_ctas == 1 and p.block_n == 256 and p.splits == 1
    # A longer K loop keeps the pair.
    p = _plan(capi, 16 * 256 * 512, 768, 256)
    assert p.cluster_ctas == 2


def test_plan_unaligned_output_disables_tma_store(capi):
    p = _plan(capi, 100, 101, 64, ldc=101)
    assert p.tma_store == 0


def test_plan_large_k_splits(capi):
    p = _plan(capi, 256, 256, 262144)
    assert p.splits > 1
    slots = p.work_units * p.cluster_ctas
    assert 100 <= slots <= 148
    assert p.kb_per_split * p.splits >= 262144 // 32


def test_plan_triangular_never_splits(capi):
    """Triangular TF32 products: CTA pairs, no split-K, one table row of units
    per CTA pair.  Untransposed operands mask through diagonal-block copies
    in workspace; transposed layouts mask inside the engine (gated transform
    warps) and need no workspace (the unit table lives in a per-device
    cache)."""
    p = _plan(capi, 256, 256, 256, op=capi.OP_TRI_UPPER)
    assert p.splits == 1 and p.cluster_ctas == 2 and p.tri_diag == 1
    assert p.workspace_bytes >= 2 * 256 * 128 * 4
    assert p.work_units % (p.grid // 2) == 0
    q = _plan(capi, 256, 256, 256, op=capi.OP_TRI_LOWER, trans_a=1)
    assert q.tri_diag == 0 and q.cluster_ctas == 2 and q.workspace_bytes == 0
    assert q.work_units % (q.grid // 2) == 0


def test_plan_irregular_stages_unaligned_operands(capi):
    p = _plan(capi, 8205, 5921, 2949)
    assert p.stage_a == 1 and p.stage_b == 1
    pitch_a = (2949 + 3) // 4 * 4
    pitch_b = (5921 + 31) // 32 * 32     # MN-major B: zero-padded to 32 columns
    exp = ((8205 * pitch_a * 4 + 255) // 256 + (2949 * pitch_b * 4 + 255) // 256) * 256
    assert p.workspace_bytes == exp
    assert capi.lib().b2g_gemm_workspace_bytes(
        ctypes.byref(capi.make_desc(8205, 5921, 2949, a=ALIGNED, b=ALIGNED, c=ALIGNED))) == exp


def test_plan_misaligned_base_pointer_is_staged(capi):
    p = _plan(capi, 256, 256, 256, a=ALIGNED + 4)
    assert p.stage_a == 1 and p.stage_b == 0


def test_plan_3xtf32_uses_narrow_tiles(capi):
    p = _plan(capi, 2048, 2048, 2048, precision=capi.PREC_3XTF32)
    assert p.block_n == 256 and p.stages == 3 and p.cluster_ctas == 2 and p.x3_split == 1
    assert p.workspace_bytes == 2 * 2048 * 2048 * 4      # lo parts of A and B


def test_plan_batched(capi):
    p = _plan(capi, 512, 2048, 1024, batch=128, stride_a=512 * 1024, stride_b=1024 * 2048,
              stride_c=512 * 2048)
    assert p.cluster_ctas == 2 and p.block_m == 256
    assert p.work_units == 2 * 8 * 128 and p.grid == 148 and p.splits == 1


@pytest.mark.parametrize("bad", [
    dict(m=-1), dict(batch=0), dict(op=7), dict(precision=5), dict(lda=3),
    dict(op=1, n=64),                     # triangular needs square
])
def test_plan_rejects_bad_descriptors(capi, bad):
    args = dict(m=128, n=128, k=128, a=ALIGNED, b=ALIGNED, c=ALIGNED)
    args.update(bad)
    m, n, k = args.pop("m"), args.pop("n"), args.pop("k")
    d = capi.make_desc(m, n, k, **args)
    p = capi.GemmPlan()
    assert capi.lib().b2g_gemm_plan_for(ctypes.byref(d), 148, ctypes.byref(p)) == \
        capi.B2G_ERR_INVALID_ARG


def test_gemm_without_gpu_reports_no_device(capi):
    import torch
    if torch.cuda.is_available():
        pytest.skip("host-only check")
    d = capi.make_desc(128, 128, 128, a=ALIGNED, b=ALIGNED, c=ALIGNED)
    assert capi.gemm(d) == capi.B2G_ERR_NO_DEVICE
