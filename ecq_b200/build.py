"""Build libecq.so in-tree (ecq_b200/_lib/libecq.so) for sm_100a with nvcc.

    python -m ecq_b200.build

The library holds the CUDA kernels, their C-ABI launchers and the host
codec; it links the CUDA runtime statically and depends on nothing else, so
it can be loaded with ctypes by any host program.
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
INCLUDE = ROOT / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libecq.so"

SOURCES = ["ecq_device.cu", "ecq_matmul.cu", "ecq_plain4.cu", "ecq_comm.cu", "ecq_glue.cu", "ecq_attention.cu", "ecq_host.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _newest_input() -> float:
    files = [CSRC / s for s in SOURCES] + list(INCLUDE.glob("*.h")) + list(CSRC.glob("*.cuh")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files if f.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if LIB.exists() and not force and LIB.stat().st_mtime >= _newest_input():
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    tmp = OUT_DIR / "_obj"
    tmp.mkdir(exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = tmp / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-pthread",
               "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if src.endswith(".cu"):
            cmd[1:1] = ["-Xptxas", "-v"] if verbose else []
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    link = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-Xcompiler", "-pthread", "-o", str(LIB) + ".tmp", *objs]
    subprocess.run(link, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="-v" in sys.argv)
    print(LIB)
