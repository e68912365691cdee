"""Build libmentat_b200.so in-tree with nvcc for sm_100a.

    python -m mentat_b200.build [--force] [-v]

The library has no torch dependency; the Python side binds it with ctypes.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libmentat_b200.so"
SOURCES = ["kv_cache.cu", "decode_attention.cu", "gate.cu", "prune.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE)]
    objs = []
    for s in SOURCES:
        o = objdir / (Path(s).stem + ".o")
        cmd = [nvcc()] + flags + ["-c", str(CSRC / s), "-o", str(o)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(o))
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc()] + ARCH + ["-shared", "-o", str(tmp)] + objs + ["-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
