"""Build libnvfp4_b200.so in-tree with nvcc for sm_100a.

    python -m nvfp4_b200.build          (from blackwell-nvfp4-kernels_b200/)

The library is self-contained (static cudart, driver entry points resolved at
run time), so it loads next to any torch build.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parent.parent / "include"
LIB_PATH = PKG_DIR / "libnvfp4_b200.so"
SOURCES = ["capi.cu"]
HEADERS = ["ptx.cuh", "kernel_common.cuh", "dual_gemm.cuh", "dual_gemm_2sm.cuh", "grouped_gemm_2sm.cuh",
           "grouped_gemm.cuh", "quantize.cuh", "moe.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
]


def nvcc_path() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "nvfp4_b200.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA library if any source is newer than the .so."""
    if not force and not _stale():
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", str(INCLUDE),
           *[str(CSRC / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr}\n{res.stdout}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
