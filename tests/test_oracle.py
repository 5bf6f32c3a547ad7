"""CPU oracle pinning: the reference's own known-answer tests, an independent
pure-Python restatement, an analytic discrete-eigenmode solution, and the
reductions of the north-star extensions to the plain reference step.

Reference tests restated here: crates/ringkernel-wavesim3d/src/simulation/
grid3d.rs:527-698 and physics.rs:675-680.
"""
import math

import numpy as np
import pytest

from rustcompute_b200 import configs
from rustcompute_b200.grid import AcousticParams3D, CellType, SimulationGrid3D


def default_params():
    # AcousticParams3D::new(Environment::default(), 0.1); the ISO band model
    # is out of scope, so the damping clamps to 1 - base_damping.
    return AcousticParams3D.new(343.0, 0.1)


def test_grid_creation():  # grid3d.rs:528-534
    g = SimulationGrid3D(32, 32, 32, default_params())
    assert (g.width, g.height, g.depth) == (32, 32, 32)
    assert g.total_cells == 32 ** 3


def test_indexing():  # grid3d.rs:537-548
    g = SimulationGrid3D(32, 32, 32, default_params())
    assert g.coords(g.index(5, 10, 15)) == (5, 10, 15)
    assert g.index(0, 0, 0) == 0
    assert g.index(31, 31, 31) == 32 ** 3 - 1


def test_impulse_injection(oracle_lib):  # grid3d.rs:551-558
    g = oracle_lib.OracleGrid(32, 32, 32, default_params())
    c = g.index(16, 16, 16)
    assert g.pressure[c] == 0.0
    g.inject_impulse_c(16, 16, 16, 1.0)
    assert g.pressure[c] == 1.0
    assert g.pressure_prev[c] == 0.5
    h = SimulationGrid3D(32, 32, 32, default_params())
    h.inject_impulse(16, 16, 16, 1.0)
    assert np.array_equal(h.pressure, g.pressure) and np.array_equal(h.pressure_prev, g.pressure_prev)


def test_wave_propagation(oracle_lib):  # grid3d.rs:561-578
    g = oracle_lib.OracleGrid(32, 32, 32, default_params())
    g.inject_impulse_c(16, 16, 16, 1.0)
    for _ in range(10):
        g.step_sequential()
    assert abs(g.pressure[g.index(17, 16, 16)]) > 0 or abs(g.pressure[g.index(16, 16, 16)]) > 0


def test_wave_spreading(oracle_lib):  # grid3d.rs:581-610
    g = oracle_lib.OracleGrid(32, 32, 32, default_params())
    g.params.simple_damping = 1.0
    g.inject_impulse_c(16, 16, 16, 1.0)
    assert g.max_pressure() > 0.5
    for _ in range(5):
        g.step_sequential()
    assert g.total_energy() > 0.0
    assert abs(g.pressure[g.index(17, 16, 16)]) > 0 or abs(g.pressure[g.index(16, 17, 16)]) > 0


def test_pressure_sampling():  # grid3d.rs:613-630
    g = SimulationGrid3D(32, 32, 32, default_params())
    g.pressure[g.index(10, 10, 10)] = 1.0
    cs = g.params.cell_size
    assert g.sample_pressure(10 * cs, 10 * cs, 10 * cs) > 0.5


def test_boundary_setup():  # grid3d.rs:633-642
    g = SimulationGrid3D(32, 32, 32, default_params())
    assert g.cell_types[g.index(0, 0, 0)] == CellType.ABSORBER
    assert g.cell_types[g.index(31, 31, 31)] == CellType.ABSORBER
    assert g.cell_types[g.index(16, 16, 16)] == CellType.NORMAL
    assert np.float32(g.reflection_coeff[g.index(0, 5, 5)]) == np.float32(0.1)


def test_boundary_setup_matches_c(oracle_lib):
    import ctypes as C
    for W, H, D in [(32, 32, 32), (13, 7, 5), (3, 3, 3), (1, 4, 2)]:
        g = SimulationGrid3D(W, H, D)
        t = np.empty(W * H * D, np.uint8)
        r = np.empty(W * H * D, np.float32)
        oracle_lib.lib().ws3o_setup_boundaries(W, H, D, t.ctypes.data, r.ctypes.data)
        assert np.array_equal(t, g.cell_types) and np.array_equal(r, g.reflection_coeff)


def test_slices():  # grid3d.rs:645-666
    g = SimulationGrid3D(32, 32, 32, default_params())
    g.pressure[g.index(5, 10, 15)] = 1.0
    xy = g.get_xy_slice(15)
    assert len(xy) == g.width * g.height and xy[10 * g.width + 5] == 1.0
    xz = g.get_xz_slice(10)
    assert len(xz) == g.width * g.depth and xz[15 * g.width + 5] == 1.0
    yz = g.get_yz_slice(5)
    assert len(yz) == g.height * g.depth and yz[15 * g.height + 10] == 1.0


def test_parallel_vs_sequential(oracle_lib):  # grid3d.rs:669-698 (bitwise here)
    a = oracle_lib.OracleGrid(16, 16, 16, default_params())
    b = oracle_lib.OracleGrid(16, 16, 16, default_params())
    a.inject_impulse_c(8, 8, 8, 1.0)
    b.inject_impulse_c(8, 8, 8, 1.0)
    for _ in range(10):
        a.step_sequential()
        b.step_parallel(4)
    assert float(np.max(np.abs(a.pressure - b.pressure))) < 1e-3
    assert np.array_equal(a.pressure, b.pressure)


def test_cfl_stability():  # physics.rs:675-680
    p = AcousticParams3D.new()
    assert p.is_stable()
    assert p.courant_number() <= 1.0 / math.sqrt(3.0) + 1e-7
    assert abs(p.c_squared - 0.25) < 1e-6


@pytest.mark.parametrize("shape,use_cells", [((7, 6, 5), False), ((9, 8, 7), True),
                                               ((5, 11, 6), False)])
def test_c_oracle_matches_python_restatement(oracle_lib, shape, use_cells):
    from oracle import pyref
    W, H, D = shape
    rng = np.random.default_rng(7)
    c2f = rng.uniform(0.02, 0.25, W * H * D).astype(np.float32)
    g = oracle_lib.OracleGrid(W, H, D, AcousticParams3D(c_squared=0.23, simple_damping=0.999),
                              c2_field=c2f, sponge_width=2, sponge_max=0.1)
    g.pressure[:] = rng.standard_normal(W * H * D).astype(np.float32)
    g.pressure_prev[:] = rng.standard_normal(W * H * D).astype(np.float32)
    if use_cells:
        g.set_cell_type(3, 3, 3, CellType.OBSTACLE)
        g.set_cell_type(4, 3, 3, CellType.REFLECTOR)
        g.set_cell_type(2, 4, 3, CellType.ABSORBER)
        g.set_cell_type(0, 2, 2, CellType.NORMAL)
    p, pp = g.pressure.copy(), g.pressure_prev.copy()
    tab = oracle_lib.sponge_table(2, 0.1)
    for _ in range(3):
        p, pp = pyref.step(W, H, D, p, pp, 0.23, 0.999,
                           types=g.cell_types if use_cells else None,
                           refl=g.reflection_coeff if use_cells else None,
                           c2_field=c2f, sponge=tab)
        g.step_sequential()
    assert np.array_equal(p, g.pressure)
    assert np.array_equal(pp, g.pressure_prev)


def test_discrete_eigenmode_known_answer(oracle_lib):
    """Analytic solution of the scheme itself: with zero faces, damping 1 and
    p = p_prev = phi (a Dirichlet eigenmode of the 7-point Laplacian with
    eigenvalue lam), the amplitude obeys A(n+1) = (2 + c2 lam) A(n) - A(n-1),
    A(0) = A(-1) = 1, so A(n) = cos(w (n + 1/2)) / cos(w / 2), cos w = 1 + c2 lam / 2."""
    W, H, D = 24, 20, 18
    a, b, c = 1, 2, 1
    kx, ky, kz = math.pi * a / (W - 1), math.pi * b / (H - 1), math.pi * c / (D - 1)
    x = np.arange(W)[None, None, :]
    y = np.arange(H)[None, :, None]
    z = np.arange(D)[:, None, None]
    phi = np.sin(kx * x) * np.sin(ky * y) * np.sin(kz * z)
    lam = (2 * math.cos(kx) - 2) + (2 * math.cos(ky) - 2) + (2 * math.cos(kz) - 2)
    c2 = 0.25
    w = math.acos(1 + c2 * lam / 2)
    g = oracle_lib.OracleGrid(W, H, D, AcousticParams3D(c_squared=c2, simple_damping=1.0))
    g.pressure[:] = phi.astype(np.float32).reshape(-1)
    g.pressure_prev[:] = g.pressure
    n = 150
    g.run(n, 1)
    expect = (math.cos(w * (n + 0.5)) / math.cos(w / 2)) * phi.reshape(-1)
    err = np.linalg.norm(g.pressure.astype(np.float64) - expect) / np.linalg.norm(expect)
    assert err < 1e-4, err


def test_extensions_reduce_to_reference(oracle_lib):
    """Uniform c2 field == scalar c2; sponge width 0 == none; zero wavelet ==
    no source: each bit for bit."""
    wl = configs.build("c1", 20, 18, 16, steps=12)
    base = oracle_lib.from_workload(wl)
    base.run(12, 1)
    g = oracle_lib.from_workload(wl)
    g.c2_field = np.full(g.total_cells, np.float32(wl.c_squared), np.float32)
    g.set_sources([[5, 5, 5], [9, 9, 9]], np.zeros((2, 12), np.float32))
    g.run(12, 1)
    assert np.array_equal(base.pressure, g.pressure)
    assert np.array_equal(base.pressure_prev, g.pressure_prev)


def test_sources_match_inject_impulse_semantic(oracle_lib):
    """A source's per-step drive equals calling inject_impulse before each step."""
    wl = configs.build("c2", 24, 24, 24, steps=30)
    g = oracle_lib.from_workload(wl)
    g.run(30, 1)
    h = oracle_lib.from_workload(wl)
    h.set_sources(np.zeros((0, 3)), None)
    for s in range(30):
        for k, (x, y, z) in enumerate(wl.sources):
            h.inject_impulse_c(int(x), int(y), int(z), float(wl.wavelet[k, s]))
        h.step_sequential()
    assert np.array_equal(g.pressure, h.pressure)


def test_sponge_table_values(oracle_lib):
    t = oracle_lib.sponge_table(16, 0.1)
    assert t[0] == np.float32(0.9)
    assert np.all(np.diff(t) > 0) and t[-1] < 1.0
    d = 5
    assert t[d] == np.float32(1.0 - np.float64(np.float32(0.1)) * ((16 - d) / 16) ** 2)


def test_persistent_config_restated():
    """persistent_backend.rs:495-513 (config defaults and builder)."""
    from rustcompute_b200 import PersistentBackendConfig
    c = PersistentBackendConfig()
    assert c.tile_size == (8, 8, 8) and c.use_cooperative and c.progress_interval == 100
    c = PersistentBackendConfig().with_tile_size(4, 4, 4).with_cooperative(False) \
        .with_progress_interval(50)
    assert c.tile_size == (4, 4, 4) and not c.use_cooperative and c.progress_interval == 50


def test_error_display_restated():
    """persistent_backend.rs:515-522 / gpu_backend.rs:13-23: error kinds and messages."""
    from rustcompute_b200 import CompileError, DeviceError, GpuError
    assert issubclass(DeviceError, GpuError) and issubclass(CompileError, GpuError)
    assert "device" in str(DeviceError("GpuBackend3D::new: GPU device error: x")).lower()
