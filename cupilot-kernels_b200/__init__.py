"""B200-native (sm_100a) fp32-input dense GEMM operator family.

A drop-in for the GEMM band (problem IDs 1-18) of champloo2878/cuPilot-Kernels:
each operator keeps the reference's Torch C++-extension entry point
`f(A, B) -> Tensor` (exported as `forward` and under the reference's own
Part-3 name, see `ops`), implemented by hand-written tcgen05/TMA kernels in
`libb2g_sm100.so` behind the C ABI in `include/b2g_gemm.h`.

There is no CPU or library fallback: importing `ops` without the built
extension raises ImportError.
"""
from __future__ import annotations

from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "libb2g_sm100.so"

__all__ = ["PACKAGE_DIR", "LIB_PATH", "native", "ops"]


def native():
    """The compiled Torch extension module (raises ImportError if unbuilt)."""
    import torch  # noqa: F401  (loads libtorch before the extension)

    try:
        from . import _b2g_torch  # type: ignore[attr-defined]
    except ImportError as e:  # pragma: no cover - exercised only when unbuilt
        raise ImportError(
            "cupilot-kernels_b200: native extension not built; run "
            "`python cupilot-kernels_b200/build.py` (nvcc, sm_100a)"
        ) from e
    return _b2g_torch


def __getattr__(name):
    if name in ("ops", "partition", "capi"):
        import importlib

        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
