"""Build the in-tree CUDA library libnvfp4_b200.so for sm_100a with nvcc.

The library is built next to this file so that it travels with the source
tree; nothing is installed into site-packages.
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
LIB = PKG / "libnvfp4_b200.so"
OBJDIR = PKG / "_build"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
SOURCES = ["rht_gemm_sm100.cu", "sr_kernels.cu", "fp8_kernels.cu", "fp8_kernels_loose.cu"]
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-v",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def _deps() -> list[Path]:
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + \
        sorted(INCLUDE.glob("*.h")) + sorted(INCLUDE.glob("*.cuh"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(d.stat().st_mtime > t for d in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    OBJDIR.mkdir(exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = OBJDIR / (Path(src).stem + ".o")
        cmd = [NVCC, *FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs, "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("link failed")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
