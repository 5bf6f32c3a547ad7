"""Resident (command-driven) persistent kernel on the GPU: ws3d_resident_*
through the PersistentBackend mirror of the reference API.

The reference drives one resident kernel with H2K commands and reads K2H
responses and a control block in mapped host memory
(persistent_backend.rs:253-446, persistent_fdtd.rs:766-978).  Checked here:
fields bit-identical to per-step runs (commands between steps, odd step
counts, sources, c2 field, sponge); PROGRESS every interval with the energy;
GET_PROGRESS echoes the command id; unknown commands answer ERROR; PAUSE /
RESUME; an idle kernel leaves after its budget and is relaunched; other
calls are refused while resident; the K2H queue drops (and counts) what does
not fit; shutdown answers TERMINATED and hands the fields back.
"""
import time

import numpy as np
import pytest

from rustcompute_b200 import (CommandError, GpuBackend3D, PersistentBackend,
                              PersistentBackendConfig, SimulationGrid3D, configs)
from rustcompute_b200 import _ffi
from rustcompute_b200.grid import AcousticParams3D
from rustcompute_b200.persistent import ResponseType

pytestmark = pytest.mark.gpu


def grids(W=96, H=40, D=36, seed=3):
    prm = AcousticParams3D(c_squared=0.2, simple_damping=0.9995)
    rng = np.random.default_rng(seed)
    a = SimulationGrid3D(W, H, D, prm)
    a.pressure[:] = rng.standard_normal(W * H * D).astype(np.float32)
    a.pressure_prev[:] = rng.standard_normal(W * H * D).astype(np.float32)
    b = SimulationGrid3D(W, H, D, prm)
    b.pressure[:] = a.pressure
    b.pressure_prev[:] = a.pressure_prev
    return a, b


def same(x, y):
    return np.array_equal(np.asarray(x).view(np.uint32), np.asarray(y).view(np.uint32))


def test_resident_equals_per_step_with_commands_between_steps():
    wl = configs.build("c3", 144, 40, 36, steps=60)
    ga, gb = grids(144, 40, 36)
    c2 = wl.c2_field()
    pb = PersistentBackend(ga, PersistentBackendConfig().with_progress_interval(7),
                           sponge_width=3, sponge_max=0.1)
    pb.backend.set_c2_field(c2)
    pb.backend.set_sources(wl.sources, wl.wavelet)
    ref = GpuBackend3D(gb, sponge_width=3, sponge_max=0.1)
    ref.set_c2_field(c2)
    ref.set_sources(wl.sources, wl.wavelet)
    for n, imp in ((13, (70, 20, 18)), (8, (1, 1, 1)), (21, (143, 39, 35)), (5, None)):
        pb.step(ga, n)
        ref.step_n(gb, n)
        if imp:
            pb.inject_impulse(*imp, 0.75)
            ref.inject_impulse(*imp, 0.75)
    pb.download_pressure(ga)
    ref.download_pressure(gb)
    assert ga.step == gb.step == 47
    assert same(ga.pressure, gb.pressure)
    st = pb.stats()
    assert st.current_step == 47 and st.steps_remaining == 0 and st.is_running
    resp = pb.poll_responses()
    prog = [r for r in resp if r[0] == ResponseType.PROGRESS]
    assert [r[1] for r in prog] == [7, 14, 21, 28, 35, 42]
    # the energy reported at step 42 is the field's sum of p^2
    pb.shutdown()
    assert pb.stats().has_terminated
    term = [r for r in pb.poll_responses() if r[0] == ResponseType.TERMINATED]
    assert len(term) == 1 and term[0][1] == 47
    e = pb.backend.energy()
    assert abs(term[0][3] - e) <= 1e-5 * e
    pb.close()
    ref.close()


def test_get_progress_unknown_command_pause_resume():
    ga, _ = grids()
    pb = PersistentBackend(ga, PersistentBackendConfig().with_progress_interval(1000))
    pb.step(ga, 4)
    pb.request_progress(cmd_id=77)
    pb.send(_ffi.WS3D_CMD_SET_SOURCE, cmd_id=78)
    deadline = time.time() + 10
    got = []
    while len(got) < 2 and time.time() < deadline:
        got += pb.poll_responses()
        time.sleep(0.001)
    kinds = {r[0] for r in got}
    assert ResponseType.PROGRESS in kinds and ResponseType.ERROR in kinds
    prog = [r for r in got if r[0] == ResponseType.PROGRESS][0]
    assert prog[1] == 4 and prog[2] == 0
    pb.pause()
    b = pb.backend
    b._chk(b._lib.ws3d_resident_run_steps(b._ctx, 5), "run_steps")
    time.sleep(0.2)
    st = pb.stats()
    assert st.current_step == 4 and st.steps_remaining == 5
    pb.resume()
    b._chk(b._lib.ws3d_resident_wait_step(b._ctx, 9, 0), "wait")
    assert pb.stats().current_step == 9
    pb.close()


def test_idle_exit_relaunch_and_calls_refused_while_resident():
    ga, gb = grids(seed=5)
    cfg = PersistentBackendConfig()
    cfg.idle_budget_s = 0.05
    pb = PersistentBackend(ga, cfg)
    ref = GpuBackend3D(gb)
    pb.step(ga, 5)
    ref.step_n(gb, 5)
    with pytest.raises(CommandError):
        pb.backend.step_n(None, 1)          # the resident kernel owns the context
    time.sleep(0.5)                          # past the idle budget: the kernel left
    st = _ffi.ws3d_resident_stats()
    b = pb.backend
    b._chk(b._lib.ws3d_resident_stats_get(b._ctx, st), "stats")
    assert st.kernel_alive == 0 and st.launches == 1 and st.is_running == 1
    pb.inject_impulse(20, 20, 20, 1.5)       # relaunches
    ref.inject_impulse(20, 20, 20, 1.5)
    pb.step(ga, 6)
    ref.step_n(gb, 6)
    b._chk(b._lib.ws3d_resident_stats_get(b._ctx, st), "stats")
    assert st.launches >= 2
    pb.download_pressure(ga)
    ref.download_pressure(gb)
    assert same(ga.pressure, gb.pressure)
    pb.shutdown()
    # the ordinary API continues from the resident run (11 steps: odd roles)
    b.step_n(None, 4)
    ref.step_n(None, 4)
    p1, pp1 = b.download_field(with_prev=True)
    p2, pp2 = ref.download_field(with_prev=True)
    assert same(p1, p2) and same(pp1, pp2) and b.stats()["step"] == 15
    pb.close()
    ref.close()


def test_k2h_overflow_is_counted_not_blocking():
    ga, _ = grids(48, 24, 20)
    cfg = PersistentBackendConfig(progress_interval=1, k2h_capacity=2)
    pb = PersistentBackend(ga, cfg)
    pb.step(ga, 10)                          # 10 PROGRESS messages, room for 2
    b = pb.backend
    st = _ffi.ws3d_resident_stats()
    b._chk(b._lib.ws3d_resident_stats_get(b._ctx, st), "stats")
    assert st.current_step == 10
    got = pb.poll_responses()
    assert len(got) == 2 and [r[1] for r in got] == [1, 2]
    pb.shutdown()
    b._chk(b._lib.ws3d_resident_stats_get(b._ctx, st), "stats")
    assert st.k2h_dropped >= 8
    pb.close()
