"""Builds libqx.so (the CUDA kernels and the C ABI of include/qx.h) for sm_100a, in-tree.

    python -m qwenputer_b200.build        # or build() from Python

nvcc compiles each source with -gencode arch=compute_100a,code=sm_100a; the library links the
CUDA runtime statically, so it loads next to any torch build.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libqx.so"
SOURCES = ["qx_exec.cu", "qx_load.cu", "qx_gdn.cu", "qx_api.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-I", str(REPO / "include"),
         "-I", str(CSRC), "--expt-relaxed-constexpr", "-static-global-template-stub=false"]


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [REPO / "include" / "qx.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    for s in SOURCES:
        o = build_dir / (Path(s).stem + ".o")
        cmd = [NVCC, *FLAGS, "-c", str(CSRC / s), "-o", str(o)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(o))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
                    *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
