"""Builds the qic shared library (qwenincuda_b200/libqic.so) for sm_100a with nvcc.

Translation units whose arithmetic must match the reference's --use_fast_math
build (the fused norm/RoPE/append/gate paths) are compiled with --use_fast_math;
the GatedDeltaNet kernel is compiled with IEEE-accurate math. Objects go to
qwenincuda_b200/_build/; a unit is rebuilt when it or a header is newer than its
object.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = PKG.parent / "include"
LIB = PKG / "libqic.so"

NVCC = os.environ.get("NVCC", "nvcc")
CXX = os.environ.get("CXX", "g++")
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]

# (source, extra flags)
UNITS = [
    ("attn_kernel.cu", ["--use_fast_math"]),
    ("rowops.cu", ["--use_fast_math"]),
    ("gdn_kernel.cu", ["--use_fast_math"]),
    ("capi.cpp", []),
    ("compat.cu", ["--use_fast_math"]),
    ("noalloc.cu", []),
    ("gemv_kernel.cu", ["--use_fast_math"]),
    ("runtime_kernels.cu", []),
    ("model_runner.cpp", []),
]


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    deps = _headers()
    objs = []
    relink = not LIB.exists()
    for name, extra in UNITS:
        src = CSRC / name
        if not src.exists():
            continue
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if _stale(obj, src, deps) or ptxas_info:
            cmd = [NVCC, *ARCH, *COMMON, *extra, "-c", str(src), "-o", str(obj)]
            if name.endswith(".cpp"):
                cmd = [CXX, "-O3", "-std=c++17", "-fPIC", "-Wall", f"-I{CUDA_HOME / 'include'}", f"-I{INCLUDE}",
                       f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
            elif ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
                raise RuntimeError(f"nvcc failed on {name}")
            if ptxas_info:
                sys.stdout.write(r.stdout + r.stderr)
            relink = True
    if relink or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-Xlinker", "-Bsymbolic", *map(str, objs), "-o", str(LIB)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link of libqic.so failed")
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas-info" in sys.argv)
    print(LIB)
