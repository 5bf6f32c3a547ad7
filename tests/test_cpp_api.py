"""The C++ mirror (include/ws3d.hpp) compiles against the C-ABI on the CPU,
and on a GPU reproduces the oracle bit for bit through GpuBackend3D and
PersistentBackend."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp_api_check.cpp")
EXE = os.path.join(ROOT, "tests", "_build", "cpp_api_check")


def build_exe():
    from rustcompute_b200 import build
    import oracle
    lib = build.build()
    olib = oracle.build()
    os.makedirs(os.path.dirname(EXE), exist_ok=True)
    libdir, olibdir = os.path.dirname(lib), os.path.dirname(olib)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"), SRC,
                    "-o", EXE, "-L", libdir, "-lws3d", os.path.join(olibdir, "libws3d_oracle.so"),
                    f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{olibdir}"], check=True)
    return EXE


def test_cpp_mirror_compiles():
    assert os.path.exists(build_exe())


@pytest.mark.gpu
def test_cpp_mirror_matches_oracle_on_gpu():
    exe = build_exe()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "CPP-API OK" in r.stdout, r.stdout + r.stderr
