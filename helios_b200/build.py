"""Builds libg4q.so (the C-ABI kernel library) in-tree with nvcc for sm_100a.

``python -m helios_b200.build`` or ``helios_b200.build.build()``. The shared library lands
next to this file so it travels with the source tree; no JIT cache is involved.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libg4q.so"
OBJDIR = PKG / "_build"

SOURCES = ["g4q_api.cu", "g4q_layout.cu", "g4q_gemv.cu", "g4q_gemv2.cu", "g4q_gemm.cu", "g4q_decode.cu",
           "g4q_generic.cu", "g4q_comm.cu", "g4q_lora.cu", "g4q_mlp.cu"]
HEADERS = ["g4q_common.cuh", "g4q_internal.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every .cu under csrc/ for sm_100a and link libg4q.so. Returns its path."""
    OBJDIR.mkdir(exist_ok=True)
    nvcc = _nvcc()
    common_deps = [CSRC / h for h in HEADERS] + [INCLUDE / "g4q.h"]
    objs, cmds = [], []
    for src in SOURCES:
        obj = OBJDIR / (src + ".o")
        objs.append(obj)
        if force or _stale(obj, [CSRC / src] + common_deps):
            cmds.append([nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(CSRC / src), "-o", str(obj)])
    # translation units compile independently: one nvcc per source, a few at a time
    from concurrent.futures import ThreadPoolExecutor

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(compile_one, cmds))
    if force or _stale(LIB, objs):
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB), *map(str, objs),
               "-lcudart", "-Xlinker", "-z,defs"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
