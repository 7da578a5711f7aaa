"""Build libcormorant_cuda.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m cormorant_b200.build [--force] [--ptxas-info]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libcormorant_cuda.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2",
                     "-I", str(INCLUDE), "-I", str(CSRC)]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, ptxas_info: bool = False, quiet: bool = True) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    objs = []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_info or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [_nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
            if not quiet:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [_nvcc(), *ARCH, "-shared", "--cudart", "static", "-o", str(LIB), *map(str, objs), "-lrt", "-ldl", "-lpthread"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_info=a.ptxas_info, quiet=False))
