"""The C-ABI library loads and exports every symbol include/ws3d.h declares.

Runs on CPU: no compute call is made.
"""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions(path):
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(ws3d_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from rustcompute_b200 import _ffi, build
    build.build()
    return _ffi.load()


def test_header_declares_expected_entry_points():
    names = header_functions(os.path.join(ROOT, "include", "ws3d.h"))
    for must in ["ws3d_create", "ws3d_destroy", "ws3d_step", "ws3d_upload", "ws3d_download",
                 "ws3d_inject_impulse", "ws3d_inject_spherical_impulse", "ws3d_energy"]:
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for hdr in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not hdr.endswith(".h"):
            continue
        for name in header_functions(os.path.join(ROOT, "include", hdr)):
            assert hasattr(lib, name), f"{name} declared in include/{hdr} but not exported"


def test_binding_table_matches_header():
    from rustcompute_b200 import _ffi
    names = header_functions(os.path.join(ROOT, "include", "ws3d.h"))
    assert sorted(_ffi.SIGNATURES) == names


def test_host_only_entry_points(lib):
    from rustcompute_b200 import _ffi
    assert lib.ws3d_abi_version() == 1
    assert lib.ws3d_status_string(_ffi.WS3D_ETIMEOUT) == b"device wait timed out"
    d = _ffi.ws3d_desc()
    lib.ws3d_desc_init(C.byref(d), 8, 9, 10)
    assert (d.width, d.height, d.depth, d.c_squared, d.damping) == (8, 9, 10, 0.25, 1.0)


def test_create_rejects_bad_desc_without_touching_device(lib):
    from rustcompute_b200 import _ffi
    d = _ffi.ws3d_desc()
    lib.ws3d_desc_init(C.byref(d), 0, 9, 10)
    ctx = C.c_void_p()
    assert lib.ws3d_create(C.byref(d), C.byref(ctx)) == _ffi.WS3D_EINVAL
    lib.ws3d_desc_init(C.byref(d), 8, 9, 10)
    d.z_begin, d.z_end = 5, 11
    assert lib.ws3d_create(C.byref(d), C.byref(ctx)) == _ffi.WS3D_EINVAL
    assert not ctx.value


def test_ctx_struct_layout():
    from rustcompute_b200 import _ffi
    assert C.sizeof(_ffi.ws3d_desc) == 56
    assert C.sizeof(_ffi.ws3d_stats) == 72
    # resident mode: the reference host's 64-byte messages (ringkernel-cuda persistent.rs)
    assert C.sizeof(_ffi.ws3d_h2k_msg) == 64
    assert C.sizeof(_ffi.ws3d_k2h_msg) == 64
    assert C.sizeof(_ffi.ws3d_resident_config) == 56
    assert C.sizeof(_ffi.ws3d_resident_stats) == 88
    # z-slab exchange: four field buffers, flags, c2 field, geometry, caps
    assert C.sizeof(_ffi.ws3d_halo_handles) == 424


def test_no_cpu_fallback_in_package():
    """The product package never imports the oracle."""
    pkg = os.path.join(ROOT, "rustcompute_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in src and "from oracle" not in src, f


def test_two_step_rows_constant_matches_the_kernel():
    """_ffi.WS3D_TWO_STEP_ROWS mirrors the default tile height in ws3d_index.h."""
    import re

    from rustcompute_b200 import _ffi
    src = open(os.path.join(ROOT, "rustcompute_b200", "csrc", "ws3d_index.h")).read()
    m = re.search(r"#define WS3D_TB_TY (\d+)", src)
    assert m and int(m.group(1)) == _ffi.WS3D_TWO_STEP_ROWS
