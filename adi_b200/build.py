"""Builds the CUDA extension of the packed MoE path in-tree, for sm_100a.

    python -m adi_b200.build

produces adi_b200/libadi_cuda.so from adi_b200/csrc/*.cu with nvcc. The
library exports the C ABI declared in include/adi_cuda.h and nothing else
(no torch types cross it).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libadi_cuda.so"
SOURCES = ["kernels.cu", "tc_gemm.cu", "ep.cu", "decode.cu", "attention.cu", "attention_tc.cu", "embedding.cu", "abi.cu", "batcher.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found")
    return found


def stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.cpp")) + [ROOT / "include" / "adi_cuda.h", Path(__file__)]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIBRARY
    out_dir = ROOT / "_build" / "adi_cuda"
    out_dir.mkdir(parents=True, exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "-I", str(ROOT / "include"), "-I", str(CSRC)]
    if verbose:
        common += ["-Xptxas", "-v"]
    objects = []
    for source in SOURCES:
        obj = out_dir / (Path(source).stem + ".o")
        cmd = common + ["-dc" if False else "-c", str(CSRC / source), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objects, "-lcudart"], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
