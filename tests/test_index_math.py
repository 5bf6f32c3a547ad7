"""CPU bounds check of the step kernels' address arithmetic.

tests/index_check.cpp is compiled with g++ against the kernel's own index
helpers (rustcompute_b200/csrc/ws3d_index.h) and replays every load and
store of the z-streaming and cp.async kernels for each launch shape below;
tests/tb_index_check.cpp replays the two-step kernel's own global accesses
(stores, stores into z-slab neighbours, loads of their edge planes) over its
launch schedule.
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


ROW_SHAPES = [(13, 7, 5), (130, 9, 20), (257, 11, 6), (3, 3, 3), (128, 128, 128), (160, 70, 37),
              (1, 1, 1), (31, 1, 2), (520, 9, 30), (256, 256, 64)]


@pytest.mark.parametrize("shape", ROW_SHAPES)
@pytest.mark.parametrize("halo,nw", [(0, 16), (1, 16), (0, 8)])
def test_persistent_row_kernel_accesses_in_bounds(checker, shape, halo, nw):
    """The block body of k_persistent_rows (16 warps) and k_resident (8): every
    access in bounds and every float4 of the owned planes written exactly once
    per step."""
    W, H, nz = shape
    r = subprocess.run([checker, str(W), str(H), str(nz), "148", str(nw), str(halo), "2"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout


SMEM_SHAPES = [(128, 128, 128), (64, 64, 64), (13, 7, 5), (3, 3, 3), (1, 1, 1), (128, 37, 29),
               (100, 130, 17), (70, 50, 41), (96, 80, 64), (128, 200, 200), (31, 1, 2)]


@pytest.mark.parametrize("shape", SMEM_SHAPES)
@pytest.mark.parametrize("c2f", [0, 1])
def test_shared_memory_persistent_kernel_indices_in_bounds(checker, shape, c2f):
    """k_persistent_smem: every shared-memory index inside its volumes, every
    global offset inside the owned planes, every row owned by one block, and
    every in-grid halo row received from exactly one neighbour's face row of
    the same global row (exchange rows inside the block's range)."""
    W, H, nz = shape
    r = subprocess.run([checker, str(W), str(H), str(nz), "148", "8", str(c2f), "3"],
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


def test_checker_catches_a_misrouted_face(tmp_path):
    """The replay of k_persistent_smem's face exchange flags a face row sent
    to the wrong exchange row of its neighbour (the mistake is planted in a
    copy of the index header)."""
    bad = tmp_path / "bad_index.h"
    src = open(os.path.join(ROOT, "rustcompute_b200", "csrc", "ws3d_index.h")).read()
    old = "        *nb = b - 1;\n        *side = 1;"
    assert src.count(old) == 1
    bad.write_text(src.replace(old, "        *nb = b - 1;\n        *side = 0;"))
    probe = tmp_path / "probe.cpp"
    probe.write_text(open(SRC).read().replace('#include "ws3d_index.h"', f'#include "{bad}"'))
    exe = tmp_path / "probe"
    subprocess.run(["g++", "-O1", "-std=c++17", "-o", str(exe), str(probe)], check=True)
    r = subprocess.run([str(exe), "64", "64", "64", "148", "8", "0", "3"], capture_output=True,
                       text=True)
    assert r.returncode == 1 and "smem xch" in r.stderr


TB_SRC = os.path.join(ROOT, "tests", "tb_index_check.cpp")
TB_BIN = os.path.join(ROOT, "tests", "_build", "tb_index_check")


@pytest.fixture(scope="module")
def tb_checker():
    os.makedirs(os.path.dirname(TB_BIN), exist_ok=True)
    inc = os.path.join(ROOT, "rustcompute_b200", "csrc")
    hdr = os.path.join(inc, "ws3d_index.h")
    if (not os.path.exists(TB_BIN) or os.path.getmtime(TB_BIN) < os.path.getmtime(TB_SRC)
            or os.path.getmtime(TB_BIN) < os.path.getmtime(hdr)):
        subprocess.run(["g++", "-O2", "-std=c++17", "-I", inc, "-o", TB_BIN, TB_SRC], check=True)
    return TB_BIN


# (W, H, nz, lower neighbour's nz, upper neighbour's nz): one GPU, first / middle / last
# slabs, two- and three-plane slabs, ragged rows and columns, the bench sizes
TB_CASES = [(512, 512, 512, 0, 0), (160, 24, 40, 0, 0), (129, 16, 3, 0, 0), (520, 17, 12, 0, 0),
            (264, 24, 23, 0, 23), (264, 24, 23, 24, 23), (264, 24, 24, 23, 0),
            (160, 40, 2, 3, 2), (160, 40, 3, 2, 2), (160, 17, 3, 2, 0), (300, 17, 30, 0, 30),
            (384, 72, 100, 100, 100), (1024, 1024, 512, 512, 0)]


@pytest.mark.parametrize("case", TB_CASES)
def test_two_step_kernel_accesses_in_bounds(tb_checker, case):
    r = subprocess.run([tb_checker, *map(str, case)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout


def test_two_step_checker_catches_a_push_one_plane_too_far(tb_checker, tmp_path):
    """Planted in a copy of the checker: the lower neighbour's second ghost
    plane addressed one plane too high must be reported."""
    src = open(TB_SRC).read()
    bad = src.replace("(int64_t)(lo_nz + qy) * P + row", "(int64_t)(lo_nz + qy + 1) * P + row")
    assert bad != src
    f = tmp_path / "tb_bad.cpp"
    f.write_text(bad)
    exe = tmp_path / "tb_bad"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I",
                    os.path.join(ROOT, "rustcompute_b200", "csrc"), "-o", str(exe), str(f)],
                   check=True)
    r = subprocess.run([str(exe), "264", "24", "23", "24", "23"], capture_output=True, text=True)
    assert r.returncode == 1 and "Y push lo" in r.stderr
