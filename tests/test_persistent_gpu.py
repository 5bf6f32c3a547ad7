"""Persistent mode (many steps in one cooperative launch) on the GPU.

Bit-identical to the per-step path and to the oracle; mixes with per-step
calls; the PersistentBackend mirror of the reference API; and the bounded
neighbour wait inside a persistent launch (a child process exports a slab
that never steps).
"""
import multiprocessing as mpm
import os
import sys
import time

import numpy as np
import pytest

import oracle
from rustcompute_b200 import (CellType, GpuBackend3D, PersistentBackend, PersistentBackendConfig,
                              ResponseType, SimulationGrid3D, TimeoutError_, configs)
from rustcompute_b200.grid import AcousticParams3D
from rustcompute_b200.slab import attach

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def backend_for(wl, variant="auto", cells=None):
    g = SimulationGrid3D(wl.W, wl.H, wl.D, AcousticParams3D(c_squared=wl.c_squared,
                                                            simple_damping=wl.damping))
    g.pressure[:], g.pressure_prev[:] = wl.initial_fields()
    if cells is not None:
        g.cell_types[:], g.reflection_coeff[:] = cells
    b = GpuBackend3D(g, variant=variant, sponge_width=wl.sponge_width, sponge_max=wl.sponge_max)
    c2 = wl.c2_field()
    if c2 is not None:
        b.set_c2_field(c2)
    if len(wl.sources):
        b.set_sources(wl.sources, wl.wavelet)
    return g, b


@pytest.mark.parametrize("name,grid,steps", [("c5", (64, 64, 64), 300),
                                             ("c3", (160, 72, 64), 90),
                                             ("c2", (96, 40, 37), 120),
                                             ("c1", (13, 7, 5), 9)])
def test_persistent_equals_step_and_oracle(name, grid, steps):
    wl = configs.build(name, *grid, steps=steps)
    _, bp = backend_for(wl)
    bp.step_persistent(steps)
    bp.sync()
    pp_, ppp = bp.download_field(with_prev=True)
    _, bs = backend_for(wl, variant="zstream")   # one launch per step
    bs.step_n(None, steps)
    sp, spp = bs.download_field(with_prev=True)
    assert np.array_equal(pp_.view(np.uint32), sp.view(np.uint32))
    assert np.array_equal(ppp.view(np.uint32), spp.view(np.uint32))
    ref = oracle.from_workload(wl)
    ref.run(steps, 1)
    assert np.array_equal(pp_.view(np.uint32), ref.pressure.view(np.uint32))


def test_persistent_with_cell_arrays():
    wl = configs.build("c1", 100, 40, 30, steps=60)
    g = SimulationGrid3D(wl.W, wl.H, wl.D)
    g.create_obstacle(20, 5, 4, 30, 12, 9, CellType.OBSTACLE)
    g.create_obstacle(60, 20, 10, 64, 25, 15, CellType.REFLECTOR)
    cells = (g.cell_types.copy(), g.reflection_coeff.copy())
    _, bp = backend_for(wl, cells=cells)
    bp.step_persistent(60)
    _, bs = backend_for(wl, variant="zstream", cells=cells)
    bs.step_n(None, 60)
    assert np.array_equal(bp.download_field(), bs.download_field())


def test_persistent_mixes_with_per_step_calls():
    wl = configs.build("c2", 70, 50, 41, steps=100)
    _, a = backend_for(wl)
    a.step_persistent(37)
    a.step_n(None, 13)
    a.step_persistent(49)
    a.step_n(None, 1)
    _, b = backend_for(wl, variant="zstream")
    b.step_n(None, 100)
    assert np.array_equal(a.download_field(), b.download_field())
    assert a.stats()["step"] == 100


@pytest.mark.parametrize("name,grid", [("c2", (96, 40, 37)), ("c3", (128, 48, 33)),
                                       ("c1", (64, 64, 64)), ("c2", (33, 17, 9)),
                                       ("c5", (128, 128, 128))])
def test_auto_multi_step_calls_on_small_grids(name, grid):
    """variant auto runs ws3d_step(n >= 2) on a small one-GPU grid as one
    persistent launch (field in shared memory) and single calls as one step
    launch; any mix of call sizes equals one launch per step bit for bit
    (sources, c2 field and sponge of the recipe)."""
    wl = configs.build(name, *grid, steps=60)
    _, a = backend_for(wl)
    _, b = backend_for(wl, variant="zstream")
    l0 = a.stats()["kernel_launches"]
    a.step_n(None, 25)
    assert a.stats()["kernel_launches"] - l0 == 1      # the 25 steps in one launch
    for n in (1, 2, 1, 7, 24):
        a.step_n(None, n)
    b.step_n(None, 60)
    pa, ppa = a.download_field(with_prev=True)
    pb, ppb = b.download_field(with_prev=True)
    assert np.array_equal(pa.view(np.uint32), pb.view(np.uint32))
    assert np.array_equal(ppa.view(np.uint32), ppb.view(np.uint32))
    assert a.stats()["step"] == 60
    a.close()
    b.close()


def test_auto_multi_step_routing_can_be_turned_off(monkeypatch):
    """WS3D_PERSISTENT_SMEM=0 at create keeps one launch per step."""
    monkeypatch.setenv("WS3D_PERSISTENT_SMEM", "0")
    wl = configs.build("c1", 64, 64, 64, steps=10)
    _, a = backend_for(wl)
    l0 = a.stats()["kernel_launches"]
    a.step_n(None, 10)
    assert a.stats()["kernel_launches"] - l0 == 10
    a.close()


def test_persistent_backend_api_restated():
    """persistent_backend.rs:253-446 behaviour through the mirror."""
    prm = AcousticParams3D.new(343.0, 0.1)
    grid = SimulationGrid3D(48, 48, 48, prm)
    grid.inject_impulse(24, 24, 24, 1.0)
    pb = PersistentBackend(grid, PersistentBackendConfig().with_progress_interval(25))
    assert not pb.is_running()
    copy = SimulationGrid3D(48, 48, 48, prm)
    pb.download_pressure(copy)                  # before start: nothing downloaded
    assert copy.total_energy() == 0.0
    pb.step(grid, 60)
    assert pb.is_running() and grid.step == 60
    st = pb.stats()
    assert st.current_step == 60 and st.steps_remaining == 0 and st.total_energy > 0
    resp = pb.poll_responses()   # PROGRESS every 25 steps, with the energy
    assert [r[1] for r in resp if r[0] == ResponseType.PROGRESS] == [25, 50]
    assert all(r[3] > 0 for r in resp) and pb.poll_responses() == []
    pb.inject_impulse(10, 10, 10, 0.5)
    pb.step(grid, 10)
    pb.download_pressure(grid)
    ref = SimulationGrid3D(48, 48, 48, prm)
    ref.inject_impulse(24, 24, 24, 1.0)
    gb = GpuBackend3D(ref)
    gb.step_n(ref, 60)
    gb.inject_impulse(10, 10, 10, 0.5)
    gb.step_n(ref, 10)
    gb.download_pressure(ref)
    assert np.array_equal(grid.pressure, ref.pressure)
    pb.shutdown()
    assert not pb.is_running() and pb.stats().has_terminated
    pb.close()


def _idle_lower_neighbour(conn, grid, zb, ze):
    sys.path.insert(0, ROOT)
    from rustcompute_b200 import GpuBackend3D as B
    from rustcompute_b200.slab import export_handles as exp
    W, H, D = grid
    b = B.create(W, H, D, z_begin=zb, z_end=ze)
    conn.send(exp(b))
    conn.recv()
    b.close()


def test_persistent_neighbour_wait_times_out():
    grid = (64, 40, 48)
    W, H, D = grid
    ctx = mpm.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_idle_lower_neighbour, args=(child, grid, 0, 24))
    proc.start()
    try:
        lower = parent.recv()
        b = GpuBackend3D.create(W, H, D, z_begin=24, z_end=48, spin_budget_ns=200_000_000)
        attach(b, lower, None)
        b._chk(b._lib.ws3d_halo_sync(b._ctx, 0), "sync0")
        b._chk(b._lib.ws3d_halo_sync(b._ctx, 1), "sync1")
        t0 = time.time()
        b.step_persistent(50)
        with pytest.raises(TimeoutError_):
            b.sync()
        assert time.time() - t0 < 30
        b.sync()
        b.close()
    finally:
        parent.send("done")
        proc.join(timeout=60)
    assert proc.exitcode == 0


@pytest.mark.parametrize("name,grid", [("c1", (64, 64, 64)), ("c3", (128, 48, 33))])
def test_small_grid_steps_allocate_nothing(name, grid):
    """The persistent shared-memory kernel's exchange rows come with the
    context (for both c2 instances): multi-step calls on a small grid, before
    and after a c2 field is set, add no device memory."""
    wl = configs.build(name, *grid, steps=20)
    _, a = backend_for(wl)          # sets the recipe's c2 field, if any
    m0 = a.memory_usage()
    a.step_n(None, 10)
    a.step_persistent(10)
    a.sync()
    assert a.memory_usage() == m0
    a.close()


@pytest.mark.parametrize("c2f", [False, True])
def test_small_grid_sources_on_block_faces(c2f):
    """Sources on the faces of the persistent kernel's blocks (64^3: blocks of
    4 rows x 8 planes; with a c2 field the shape may differ, so rows and planes
    around every multiple of 4 and 8 are covered), coinciding pairs included:
    each block applies them to its cells and to its halo copies, and the
    result equals one launch per step bit for bit."""
    W = H = D = 64
    rng = np.random.default_rng(11)
    pts = [[x, y, z] for x in (1, 31, 62) for y in (3, 4, 7, 8, 31, 32) for z in (7, 8, 15, 16, 40)]
    pts = np.array(pts[:60] + pts[:3], np.uint32)          # three coinciding pairs
    wav = rng.standard_normal((len(pts), 40)).astype(np.float32)
    c2 = rng.uniform(0.01, 0.25, W * H * D).astype(np.float32) if c2f else None
    runs = []
    for variant in ("auto", "zstream"):
        g = SimulationGrid3D(W, H, D, AcousticParams3D(c_squared=0.2, simple_damping=0.999))
        b = GpuBackend3D(g, variant=variant, sponge_width=4, sponge_max=0.1)
        if c2 is not None:
            b.set_c2_field(c2)
        b.set_sources(pts, wav)
        b.step_n(None, 37)
        runs.append(b.download_field(with_prev=True))
        b.close()
    (pa, ppa), (pb, ppb) = runs
    assert float(np.max(np.abs(pb))) > 1e-6
    assert np.array_equal(pa.view(np.uint32), pb.view(np.uint32))
    assert np.array_equal(ppa.view(np.uint32), ppb.view(np.uint32))
