"""PersistentBackend: a resident kernel driven by commands, mirroring the
reference API.

Reference: crates/ringkernel-wavesim3d/src/simulation/persistent_backend.rs
(config :86-131, stats :133-167, backend :174-446) over ringkernel-cuda
persistent.rs.  As there, one kernel stays on the GPU and is driven through
queues in pinned mapped host memory: `step` sends RUN_STEPS and polls the
control block until the kernel reports the target step (10 s timeout),
`inject_impulse` sends INJECT_IMPULSE, `poll_responses` drains the
kernel-to-host queue (PROGRESS every progress_interval steps, with the
energy), `shutdown` sends TERMINATE.  The C-ABI is ws3d_resident_*.  The
kernel runs the same cell body as GpuBackend3D.step_n, so fields are
bit-identical.  Its waits are bounded: an idle kernel leaves after
idle_budget_s and is relaunched by the next call that has work for it.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import ctypes as C

import numpy as np

from . import _ffi
from .backend import GpuBackend3D
from .grid import SimulationGrid3D


@dataclass
class PersistentBackendConfig:
    """persistent_backend.rs:86-131.  tile_size and use_cooperative are
    accepted for API compatibility (the kernel picks its own tiling: 128 x 8
    cells per CTA row block, z-chunks balanced over the co-resident CTAs; the
    launch is always cooperative).  Queue capacities are powers of two."""

    tile_size: Tuple[int, int, int] = (8, 8, 8)
    use_cooperative: bool = True
    progress_interval: int = 100
    h2k_capacity: int = 256
    k2h_capacity: int = 256
    idle_budget_s: float = 1.0

    def with_tile_size(self, tx: int, ty: int, tz: int) -> "PersistentBackendConfig":
        self.tile_size = (tx, ty, tz)
        return self

    def with_cooperative(self, use_coop: bool) -> "PersistentBackendConfig":
        self.use_cooperative = use_coop
        return self

    def with_progress_interval(self, interval: int) -> "PersistentBackendConfig":
        self.progress_interval = interval
        return self


class ResponseType(enum.IntEnum):
    """K2H response kinds (persistent.rs ResponseType, persistent_backend.rs:408-414)."""

    ACK = 0
    PROGRESS = 1
    ERROR = 2
    TERMINATED = 3
    ENERGY = 4


@dataclass
class PersistentBackendStats:
    """persistent_backend.rs:133-152."""

    current_step: int = 0
    steps_remaining: int = 0
    total_energy: float = 0.0
    messages_processed: int = 0
    k2k_sent: int = 0
    k2k_received: int = 0
    has_terminated: bool = False
    is_running: bool = False


class PersistentBackend:
    def __init__(self, grid: SimulationGrid3D,
                 config: Optional[PersistentBackendConfig] = None, *, device: int = 0,
                 sponge_width: int = 0, sponge_max: float = 0.0):
        """persistent_backend.rs:187-248: device state for `grid`."""
        self.config = config or PersistentBackendConfig()
        self._gpu = GpuBackend3D(grid, device=device, variant="zstream",
                                 sponge_width=sponge_width, sponge_max=sponge_max)
        self.started = False

    @property
    def backend(self) -> GpuBackend3D:
        return self._gpu

    def _chk(self, st: int, what: str) -> None:
        self._gpu._chk(st, what)

    def start(self) -> None:
        """persistent_backend.rs:253-264: launch the resident kernel."""
        if self.started:
            return
        c = self.config
        cfg = _ffi.ws3d_resident_config(progress_interval=int(c.progress_interval),
                                        h2k_capacity=int(c.h2k_capacity),
                                        k2h_capacity=int(c.k2h_capacity),
                                        idle_budget_ns=int(c.idle_budget_s * 1e9))
        b = self._gpu
        self._chk(b._lib.ws3d_resident_start(b._ctx, C.byref(cfg)), "PersistentBackend::start")
        self.started = True

    def send(self, cmd: int, *, cmd_id: int = 0, param1: int = 0, param2: int = 0,
             param3: int = 0, param4: float = 0.0, param5: float = 0.0) -> None:
        """Enqueue one H2K command (persistent_fdtd.rs:257-264 codes)."""
        if not self.started:
            self.start()
        m = _ffi.ws3d_h2k_msg(cmd=cmd, cmd_id=cmd_id, param1=param1, param2=param2,
                              param3=param3, param4=param4, param5=param5)
        b = self._gpu
        self._chk(b._lib.ws3d_resident_send(b._ctx, C.byref(m)), "PersistentBackend::send")

    def step(self, grid: SimulationGrid3D, steps: int, timeout_s: float = 10.0) -> None:
        """persistent_backend.rs:269-336: RUN_STEPS, then wait for the kernel
        to report the target step (10 s timeout like the reference)."""
        if not self.started:
            self.start()
        b = self._gpu
        target = self.stats().current_step + int(steps)
        self._chk(b._lib.ws3d_resident_run_steps(b._ctx, int(steps)), "PersistentBackend::step")
        self._chk(b._lib.ws3d_resident_wait_step(b._ctx, target, int(timeout_s * 1e9)),
                  "PersistentBackend::step")
        grid.advance_clock(steps)

    def inject_impulse(self, x: int, y: int, z: int, amplitude: float) -> None:
        """persistent_backend.rs:339-356 (INJECT_IMPULSE; p += a, p_prev += a/2)."""
        if not self.started:
            self.start()
        b = self._gpu
        self._chk(b._lib.ws3d_resident_inject_impulse(b._ctx, x, y, z, np.float32(amplitude)),
                  "PersistentBackend::inject_impulse")

    def pause(self) -> None:
        self.send(_ffi.WS3D_CMD_PAUSE)

    def resume(self) -> None:
        self.send(_ffi.WS3D_CMD_RESUME)

    def request_progress(self, cmd_id: int = 0) -> None:
        """GET_PROGRESS: the kernel answers with a PROGRESS message."""
        self.send(_ffi.WS3D_CMD_GET_PROGRESS, cmd_id=cmd_id)

    def reset(self, grid: SimulationGrid3D) -> None:
        """persistent_backend.rs:359-367 shuts the kernel down; here the device
        state is also reloaded from `grid` so the next step starts from it."""
        self.shutdown()
        self._gpu.reset(grid)

    def download_pressure(self, grid: SimulationGrid3D, timeout_s: float = 10.0) -> None:
        """persistent_backend.rs:370-393 (nothing to download before start):
        waits until the kernel ran every requested step, copies while it stays
        resident."""
        if not self.started:
            return
        out = np.empty(self._gpu.n_local, dtype=np.float32)
        b = self._gpu
        self._chk(b._lib.ws3d_resident_download(b._ctx, out.ctypes.data_as(C.POINTER(C.c_float)),
                                                int(timeout_s * 1e9)),
                  "PersistentBackend::download_pressure")
        grid.pressure[:] = out

    def stats(self) -> PersistentBackendStats:
        """persistent_backend.rs:396-400 (the mapped control block)."""
        st = _ffi.ws3d_resident_stats()
        b = self._gpu
        self._chk(b._lib.ws3d_resident_stats_get(b._ctx, C.byref(st)), "PersistentBackend::stats")
        return PersistentBackendStats(current_step=int(st.current_step),
                                      steps_remaining=int(st.steps_remaining),
                                      total_energy=float(st.total_energy),
                                      messages_processed=int(st.messages_processed),
                                      has_terminated=bool(st.has_terminated),
                                      is_running=self.started and bool(st.is_running))

    def poll_responses(self) -> List[tuple]:
        """persistent_backend.rs:403-419: (type, step, steps_remaining, energy)."""
        buf = (_ffi.ws3d_k2h_msg * 256)()
        n = C.c_uint32(0)
        out: List[tuple] = []
        b = self._gpu
        while True:
            self._chk(b._lib.ws3d_resident_poll(b._ctx, buf, 256, C.byref(n)),
                      "PersistentBackend::poll_responses")
            for k in range(n.value):
                m = buf[k]
                t = m.resp_type
                out.append((ResponseType(t) if t <= 4 else ResponseType.ACK, int(m.step),
                            int(m.steps_remaining), float(m.energy)))
            if n.value < 256:
                return out

    def shutdown(self) -> None:
        """persistent_backend.rs:422-433: TERMINATE and wait for the kernel."""
        if not self.started:
            return
        b = self._gpu
        self.started = False
        self._chk(b._lib.ws3d_resident_shutdown(b._ctx, 0), "PersistentBackend::shutdown")

    def is_running(self) -> bool:
        return self.started and self.stats().is_running

    def close(self) -> None:
        try:
            self.shutdown()
        finally:
            self._gpu.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
