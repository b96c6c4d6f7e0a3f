"""Build libnsnkv.so (sm_100a) in-tree with nvcc.

    python -m nsn_b200.build          # rebuild if any source is newer than the .so

The library is a plain C-ABI shared object (include/nsnkv.h); the CUDA runtime
is linked statically, so the .so only needs the NVIDIA driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libnsnkv.so"
SOURCES = ["codec.cu", "attention.cu", "int3asym.cu", "scores.cu", "paged_step.cu", "model.cu", "peer_merge.cu"]
HEADERS = ["nsnkv_common.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "nsnkv.h", Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-shared",
           "-I", str(ROOT / "include"), *[str(CSRC / s) for s in SOURCES], "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
