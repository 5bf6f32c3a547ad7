"""CPU bounds check of the step kernel's address arithmetic.

tests/index_check.cpp is compiled with g++ against the kernel's own index
helpers (rustcompute_b200/csrc/ws3d_index.h) and replays every load and
store of the z-streaming kernel for each launch shape below.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "index_check.cpp")
BIN = os.path.join(ROOT, "tests", "_build", "index_check")


@pytest.fixture(scope="module")
def checker():
    os.makedirs(os.path.dirname(BIN), exist_ok=True)
    inc = os.path.join(ROOT, "rustcompute_b200", "csrc")
    hdr = os.path.join(inc, "ws3d_index.h")
    if (not os.path.exists(BIN) or os.path.getmtime(BIN) < os.path.getmtime(SRC)
            or os.path.getmtime(BIN) < os.path.getmtime(hdr)):
        subprocess.run(["g++", "-O2", "-std=c++17", "-I", inc, "-o", BIN, SRC], check=True)
    return BIN


SHAPES = [(13, 7, 5), (33, 17, 9), (130, 9, 20), (257, 11, 6), (3, 3, 3), (4, 40, 3),
          (160, 70, 37), (40, 36, 34), (64, 64, 64), (1, 1, 1), (31, 1, 2), (96, 72, 64),
          (70, 33, 21), (48, 44, 40), (128, 128, 128), (256, 256, 256), (512, 512, 512),
          (512, 512, 64), (1024, 1024, 128), (1024, 1024, 1024), (520, 9, 300)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("sms,halo", [(148, 0), (1, 0), (148, 1)])
def test_zstream_accesses_in_bounds(checker, shape, sms, halo):
    W, H, nz = shape
    r = subprocess.run([checker, str(W), str(H), str(nz), str(sms), "8", str(halo)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout


ASYNC_SHAPES = [(13, 7, 5), (130, 9, 20), (257, 11, 6), (3, 3, 3), (160, 70, 37), (40, 36, 34),
                (64, 64, 64), (512, 512, 64), (520, 17, 300), (256, 256, 256)]


@pytest.mark.parametrize("shape", ASYNC_SHAPES)
@pytest.mark.parametrize("halo", [0, 1])
def test_async_kernel_accesses_in_bounds(checker, shape, halo):
    W, H, nz = shape
    r = subprocess.run([checker, str(W), str(H), str(nz), "148", "8", str(halo), "1"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout


def test_checker_catches_the_unsigned_wrap(checker, tmp_path):
    """The check must flag the bug class it exists for: a ghost-plane offset
    computed in uint32 (zb - 1 wrapping to 2^32 - 1)."""
    bad = tmp_path / "bad_index.h"
    src = open(os.path.join(ROOT, "rustcompute_b200", "csrc", "ws3d_index.h")).read()
    src = src.replace("WS3D_HD int64_t zs_plane(int64_t z, int64_t plane) { return z * plane; }",
                      "WS3D_HD int64_t zs_plane(int64_t z, int64_t plane) "
                      "{ return (int64_t)(uint32_t)z * plane; }")
    assert "(uint32_t)z" in src
    bad.write_text(src)
    probe = tmp_path / "probe.cpp"
    probe.write_text(open(SRC).read().replace('#include "ws3d_index.h"', f'#include "{bad}"'))
    exe = tmp_path / "probe"
    subprocess.run(["g++", "-O1", "-std=c++17", "-o", str(exe), str(probe)], check=True)
    r = subprocess.run([str(exe), "40", "36", "34", "148"], capture_output=True, text=True)
    assert r.returncode == 1 and "OUT OF BOUNDS" in r.stderr
