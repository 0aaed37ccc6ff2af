"""Build recipe for libouroq.so (the C-ABI library) with nvcc for sm_100a.

Usage: python -m ouroboros_b200.build  [--force]

The library is built in-tree (ouroboros_b200/libouroq.so) so that it travels
with the repository snapshot to the GPU box. Object files go to
ouroboros_b200/_build/ and are rebuilt only when a source is newer.
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
BUILD = PKG / "_build"
LIB = PKG / "libouroq.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "-Xptxas", "-warn-spills", "--threads", "0", "-I", str(ROOT / "include"),
              "-I", str(CSRC)]
CU_SOURCES = ["quant.cu", "gemv.cu", "gemv_stream.cu", "repack.cu", "gemm_tc.cu", "gemm_sign_tc.cu", "noalloc.cu", "shard.cu", "refmt.cu", "decode.cu",
              "head.cu"]
CPP_SOURCES = ["api.cpp", "bmts.cpp"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found")
    return exe


def _headers() -> list[Path]:
    return list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "ouroq.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *_headers()])


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    objs = []
    for name in CU_SOURCES + CPP_SOURCES:
        src = CSRC / name
        if not src.exists():
            continue
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if force or _stale(obj, src):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if name.endswith(".cpp"):
                cmd = [nvcc(), "-x", "cu", *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs),
               "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def ptxas_report() -> str:
    """Register / spill / shared-memory report of every kernel (nvcc -Xptxas -v)."""
    out = []
    for name in CU_SOURCES:
        src = CSRC / name
        if not src.exists():
            continue
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o", os.devnull]
        r = subprocess.run(cmd, capture_output=True, text=True)
        out.append(r.stderr)
    return "\n".join(out)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    if "--ptxas" in sys.argv:
        print(ptxas_report())
