"""Build libws3d.so (CUDA kernels + C-ABI) in-tree for sm_100a.

Usage: python -m rustcompute_b200.build [-v]

The library is written next to this file (rustcompute_b200/_lib/libws3d.so)
so that it travels with the source tree; no JIT cache is involved.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libws3d.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    # Every stencil multiply/add is an explicit *_rn intrinsic already; keep
    # the rest of the file free of contraction too.
    "--fmad=false",
    # host code too: the volume renderer's camera basis is recomputed bit for
    # bit by the CPU restatement
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden,-ffp-contract=off",
    "-shared",
]
SOURCES = ["ws3d_api.cu", "ws3d_noalloc.cu"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libws3d.so")


def _host_compiler_flags() -> list[str]:
    # Use the system g++ (the toolchain nvcc 12.9 supports), not a CXX override.
    gxx = shutil.which("g++", path="/usr/bin") or shutil.which("g++")
    return ["-ccbin", gxx] if gxx else []


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    deps.append(os.path.join(INCLUDE, "ws3d.h"))
    if os.path.exists(LIB) and not ptxas_verbose:
        lib_mtime = os.path.getmtime(LIB)
        if all(os.path.getmtime(d) <= lib_mtime for d in deps):
            return LIB
    cmd = [nvcc_path(), *ARCH, *NVCC_FLAGS, *_host_compiler_flags(), "-I", INCLUDE, "-I", CSRC]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB + ".tmp"
    cmd += ["-o", tmp, *srcs]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_verbose:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(verbose=v, ptxas_verbose="--ptxas" in sys.argv))
