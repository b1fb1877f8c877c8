"""Build recipe for the package's native code, in-tree.

Produces, next to this file:
  libb2g_sm100.so           the C-ABI library (include/b2g_gemm.h): the
                            tcgen05 GEMM engine, the row-scale kernel and the
                            host dispatcher; nvcc, sm_100a only, no torch.
  _b2g_torch<ext-suffix>    the Torch C++ extension (forward(A, B) per
                            operator) linked against libb2g_sm100.so.

Rebuilds only what is older than its sources.  nvcc cross-compiles here
without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = PKG / "libb2g_sm100.so"
EXT = PKG / ("_b2g_torch" + sysconfig.get_config_var("EXT_SUFFIX"))

CU_SOURCES = [CSRC / "b2g_capi.cu", CSRC / "b2g_vector.cu", CSRC / "b2g_peer.cu"]
CU_DEPS = CU_SOURCES + [CSRC / "gemm_engine.cuh", CSRC / "sdpa_engine.cuh", CSRC / "ptx_sm100.cuh",
                        CSRC / "b2g_internal.h",
                        INCLUDE / "b2g_gemm.h"]
EXT_SOURCES = [CSRC / "torch_binding.cpp"]


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_lib(verbose: bool = False, force: bool = False) -> Path:
    if force or _stale(LIB, CU_DEPS):
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
               "-Xcompiler", "-fvisibility=hidden", "-shared", "-I", INCLUDE,
               "-o", LIB, *CU_SOURCES]
        _run(cmd, verbose)
    return LIB


def build_ext(verbose: bool = False, force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension as ce

    build_lib(verbose, force)
    if force or _stale(EXT, EXT_SOURCES + [LIB, INCLUDE / "b2g_gemm.h"]):
        incs = ce.include_paths() + [sysconfig.get_paths()["include"], str(CUDA_HOME / "include"),
                                     str(INCLUDE)]
        torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_b2g_torch",
               "-DTORCH_API_INCLUDE_EXTENSION_H"]
        cmd += [f"-I{i}" for i in incs]
        cmd += [*EXT_SOURCES, "-o", EXT, f"-L{torch_lib}", f"-L{PKG}", "-lb2g_sm100",
                "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
                "-ltorch_python", f"-L{CUDA_HOME / 'lib64'}", "-lcudart",
                "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
        _run(cmd, verbose)
    return EXT


def build(verbose: bool = False, force: bool = False) -> None:
    build_ext(verbose, force)


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
