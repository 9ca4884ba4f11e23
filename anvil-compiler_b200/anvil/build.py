"""Build libanvil_cuda.so in-tree with nvcc (sm_100a only).

    python -m anvil.build            # or anvil.build.build(); __graft_entry__.build() calls it

One translation unit (csrc/anvil_abi.cu includes every kernel header) compiled with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`, the CUDA runtime linked statically, and no link-time
dependency on libcuda (driver entry points are fetched at run time), so the library also loads on a machine
without a GPU driver (the CPU test suite checks its exported symbols there).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parents[1] / "include"
LIB = PKG / "_lib" / "libanvil_cuda.so"
SOURCES = ["anvil_abi.cu"]
HEADERS = ["common.cuh", "gemm.cuh", "rowops.cuh", "attention.cuh"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found (set $NVCC)")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS if (CSRC / h).exists()]
    deps.append(INCLUDE / "anvil_cuda.h")
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of libanvil_cuda.so."""
    if not force and not ptxas_verbose and not _stale():
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
           "--shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-I", str(INCLUDE),
           "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(CSRC / s) for s in SOURCES] + ["-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stderr[-8000:]}")
    if ptxas_verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv))
