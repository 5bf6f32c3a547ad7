"""ws3d_field_energy_static: the energy reduction for callers that cannot
allocate device memory (real-time loops that must not block on cudaMalloc,
hosts that own all device memory).  Its scratch is a fixed device array inside
the library; the caller passes the field and the result slot.

Checked against the existing entry point (ws3d_energy, which reduces through
scratch allocated at context creation) on two calls in a row, with the
tolerance the other energy test uses (1e-12 relative: both accumulate in f64,
in different orders).  This file is collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

from rustcompute_b200 import GpuBackend3D, SimulationGrid3D, _ffi, configs
from rustcompute_b200.grid import AcousticParams3D

pytestmark = pytest.mark.gpu
REL = 1e-12


def static_energy(lib, field_ptr, W, H, nz, pitch, result_ptr, stream):
    err = C.create_string_buffer(256)
    st = lib.ws3d_field_energy_static(C.c_void_p(field_ptr), W, H, nz, pitch,
                                      C.c_void_p(result_ptr), C.c_void_p(stream), err, 256)
    return st, err.value.decode()


def test_static_energy_matches_ws3d_energy_twice():
    import torch
    lib = _ffi.load()
    wl = configs.build("c1", 48, 40, 36, steps=0)
    g = SimulationGrid3D(wl.W, wl.H, wl.D, AcousticParams3D(c_squared=0.25, simple_damping=1.0))
    g.pressure[:], g.pressure_prev[:] = wl.initial_fields()
    b = GpuBackend3D(g)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    result = torch.zeros(1, dtype=torch.float64, device=dev)
    W, H, D = wl.W, wl.H, wl.D
    for call, (steps, pitch) in enumerate([(17, W), (40, W + 13)]):
        b.step_n(None, steps)
        ref = b.energy()                          # existing entry point
        p = b.download_field()
        buf = torch.full((D, H, pitch), float("nan"), dtype=torch.float32, device=dev)
        buf[:, :, :W] = torch.from_numpy(p.reshape(D, H, W)).to(dev)
        result.fill_(-1.0)
        st, msg = static_energy(lib, buf.data_ptr(), W, H, D, pitch, result.data_ptr(),
                                stream.cuda_stream)
        assert st == _ffi.WS3D_OK, msg
        torch.cuda.synchronize(dev)
        got = float(result.item())
        assert abs(got - ref) <= REL * max(abs(ref), 1.0), (call, got, ref)
        want = float(np.dot(p.astype(np.float64), p.astype(np.float64)))
        assert abs(got - want) <= REL * max(want, 1.0)
    b.close()


def test_static_energy_rejects_too_many_planes():
    import torch
    lib = _ffi.load()
    dev = torch.device("cuda", 0)
    field = torch.zeros(64, dtype=torch.float32, device=dev)
    result = torch.zeros(1, dtype=torch.float64, device=dev)
    limit = int(_ffi.WS3D_STATIC_ENERGY_MAX_PLANES)
    st, msg = static_energy(lib, field.data_ptr(), 8, 8, limit + 1, 8, result.data_ptr(), 0)
    assert st == _ffi.WS3D_EINVAL
    assert str(limit) in msg and "planes" in msg
