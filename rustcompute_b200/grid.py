"""Host-side simulation grid, mirroring SimulationGrid3D.

Reference: crates/ringkernel-wavesim3d/src/simulation/grid3d.rs (struct
:29-61, new/setup_boundaries :71-116, index/coords :120-132, injection
:146-191, cell types :193-219, slices :413-442, energy :445-455, reset
:458-463) and physics.rs:459-486 (AcousticParams3D::new).

This object only holds host arrays.  It has no step method: stepping is the
GPU backend's job (GpuBackend3D / PersistentBackend), and there is no CPU
fallback in this package.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass

import numpy as np


class CellType(enum.IntEnum):
    """grid3d.rs:11-23; discriminants as uploaded by gpu_backend.rs:261-270."""

    NORMAL = 0
    ABSORBER = 1
    REFLECTOR = 2
    OBSTACLE = 3


@dataclass
class AcousticParams3D:
    """Scalar parameters the step uses (physics.rs:427-442)."""

    speed_of_sound: float = 343.0
    cell_size: float = 0.1
    time_step: float = 0.0
    c_squared: float = 0.25
    simple_damping: float = 1.0

    @classmethod
    def new(cls, speed_of_sound: float = 343.0, cell_size: float = 0.1,
            average_damping: float = 0.0, base_damping: float = 0.0001) -> "AcousticParams3D":
        """physics.rs:459-486 evaluated in f32: dt = dx/(2c), Courant^2 =
        (c*dt/dx)^2, simple_damping = clamp(1 - max(avg, base), 0.99, 0.9999).
        The ISO 9613-1 band model that yields `average_damping` is host-side
        and out of scope; pass its value."""
        f = np.float32
        speed = f(speed_of_sound)
        dx = f(cell_size)
        dt = f(dx / (speed * f(2.0)))
        courant = f(f(speed * dt) / dx)
        c2 = f(courant * courant)
        damp = f(f(1.0) - max(f(average_damping), f(base_damping)))
        damp = f(min(max(damp, f(0.99)), f(0.9999)))
        return cls(float(speed), float(dx), float(dt), float(c2), float(damp))

    def courant_number(self) -> float:
        return float(np.sqrt(np.float32(self.c_squared)))

    def is_stable(self) -> bool:
        """physics.rs:511-513."""
        return self.courant_number() <= float(np.float32(1.0) / np.sqrt(np.float32(3.0)))


class SimulationGrid3D:
    """z-major SoA grid: index = z*W*H + y*W + x (grid3d.rs:120-122)."""

    def __init__(self, width: int, height: int, depth: int,
                 params: AcousticParams3D | None = None):
        if width <= 0 or height <= 0 or depth <= 0:
            raise ValueError("grid dimensions must be positive")
        self.width, self.height, self.depth = int(width), int(height), int(depth)
        self.params = params if params is not None else AcousticParams3D()
        n = self.width * self.height * self.depth
        self.total_cells = n
        self.slice_size = self.width * self.height
        self.pressure = np.zeros(n, dtype=np.float32)
        self.pressure_prev = np.zeros(n, dtype=np.float32)
        self.cell_types = np.zeros(n, dtype=np.uint8)
        self.reflection_coeff = np.ones(n, dtype=np.float32)
        self.step = 0
        self.time = np.float32(0.0)
        self._setup_boundaries()

    def _setup_boundaries(self) -> None:
        """grid3d.rs:96-116: every face cell Absorber with reflection 0.1."""
        W, H, D = self.width, self.height, self.depth
        t = self.cell_types.reshape(D, H, W)
        r = self.reflection_coeff.reshape(D, H, W)
        for sl in (np.s_[0, :, :], np.s_[D - 1, :, :], np.s_[:, 0, :], np.s_[:, H - 1, :],
                   np.s_[:, :, 0], np.s_[:, :, W - 1]):
            t[sl] = CellType.ABSORBER
            r[sl] = np.float32(0.1)

    # -- indexing (grid3d.rs:120-143) ---------------------------------------
    def index(self, x: int, y: int, z: int) -> int:
        return z * self.slice_size + y * self.width + x

    def coords(self, idx: int) -> tuple[int, int, int]:
        z, rem = divmod(idx, self.slice_size)
        y, x = divmod(rem, self.width)
        return x, y, z

    def in_bounds(self, x: int, y: int, z: int) -> bool:
        return 0 <= x < self.width and 0 <= y < self.height and 0 <= z < self.depth

    # -- host-side edits (grid3d.rs:146-219) ----------------------------------
    def inject_impulse(self, x: int, y: int, z: int, amplitude: float) -> None:
        if x < self.width and y < self.height and z < self.depth:
            i = self.index(x, y, z)
            a = np.float32(amplitude)
            self.pressure[i] = np.float32(self.pressure[i] + a)
            self.pressure_prev[i] = np.float32(self.pressure_prev[i] + np.float32(a * np.float32(0.5)))

    def set_cell_type(self, x: int, y: int, z: int, cell_type: CellType) -> None:
        if x < self.width and y < self.height and z < self.depth:
            i = self.index(x, y, z)
            self.cell_types[i] = int(cell_type)
            self.reflection_coeff[i] = {
                CellType.NORMAL: 1.0, CellType.ABSORBER: 0.0,
                CellType.REFLECTOR: 1.0, CellType.OBSTACLE: 0.8}[CellType(cell_type)]

    def create_obstacle(self, x0: int, y0: int, z0: int, x1: int, y1: int, z1: int,
                        cell_type: CellType) -> None:
        """grid3d.rs:208-219 with the corners already in grid indices."""
        for z in range(z0, min(z1, self.depth - 1) + 1):
            for y in range(y0, min(y1, self.height - 1) + 1):
                for x in range(x0, min(x1, self.width - 1) + 1):
                    self.set_cell_type(x, y, z, cell_type)

    def has_default_cells(self) -> bool:
        """True when cell_types / reflection_coeff hold the setup_boundaries
        layout (interior Normal, faces Absorber with reflection 0.1)."""
        W, H, D = self.width, self.height, self.depth
        t = self.cell_types.reshape(D, H, W)
        r = self.reflection_coeff.reshape(D, H, W)
        if t[1:-1, 1:-1, 1:-1].any():
            return False
        tenth = np.float32(0.1)
        for sl in (np.s_[0, :, :], np.s_[D - 1, :, :], np.s_[:, 0, :], np.s_[:, H - 1, :],
                   np.s_[:, :, 0], np.s_[:, :, W - 1]):
            if not (np.all(t[sl] == CellType.ABSORBER) and np.all(r[sl] == tenth)):
                return False
        return True

    # -- readback helpers (grid3d.rs:372-455) ----------------------------------
    def sample_pressure(self, px: float, py: float, pz: float) -> float:
        """Trilinear interpolation at a position in metres (grid3d.rs:373-411), f32."""
        f = np.float32
        cs = f(self.params.cell_size)
        fx, fy, fz = f(f(px) / cs), f(f(py) / cs), f(f(pz) / cs)
        x0, y0, z0 = int(np.floor(fx)), int(np.floor(fy)), int(np.floor(fz))
        x1, y1, z1 = min(x0 + 1, self.width - 1), min(y0 + 1, self.height - 1), min(z0 + 1, self.depth - 1)
        tx, ty, tz = f(fx - f(x0)), f(fy - f(y0)), f(fz - f(z0))
        P = self.pressure
        c000, c100 = P[self.index(x0, y0, z0)], P[self.index(x1, y0, z0)]
        c010, c110 = P[self.index(x0, y1, z0)], P[self.index(x1, y1, z0)]
        c001, c101 = P[self.index(x0, y0, z1)], P[self.index(x1, y0, z1)]
        c011, c111 = P[self.index(x0, y1, z1)], P[self.index(x1, y1, z1)]
        one = f(1.0)
        lerp = lambda a, b, t: f(f(a * f(one - t)) + f(b * t))  # noqa: E731
        c00, c01 = lerp(c000, c100, tx), lerp(c001, c101, tx)
        c10, c11 = lerp(c010, c110, tx), lerp(c011, c111, tx)
        c0, c1 = lerp(c00, c10, ty), lerp(c01, c11, ty)
        return float(lerp(c0, c1, tz))

    def field(self) -> np.ndarray:
        return self.pressure.reshape(self.depth, self.height, self.width)

    def get_xy_slice(self, z: int) -> np.ndarray:
        z = min(z, self.depth - 1)
        s = z * self.slice_size
        return self.pressure[s:s + self.slice_size].copy()

    def get_xz_slice(self, y: int) -> np.ndarray:
        y = min(y, self.height - 1)
        return self.field()[:, y, :].reshape(-1).copy()

    def get_yz_slice(self, x: int) -> np.ndarray:
        x = min(x, self.width - 1)
        return self.field()[:, :, x].reshape(-1).copy()

    def total_energy(self) -> float:
        """Sum of p^2 (accumulated in f64; the reference sums in f32)."""
        p = self.pressure.astype(np.float64)
        return float(np.dot(p, p))

    def max_pressure(self) -> float:
        return float(np.max(np.abs(self.pressure))) if self.total_cells else 0.0

    def reset(self) -> None:
        self.pressure.fill(0)
        self.pressure_prev.fill(0)
        self.step = 0
        self.time = np.float32(0.0)

    def dimensions(self) -> tuple[int, int, int]:
        return self.width, self.height, self.depth

    def physical_size(self) -> tuple[float, float, float]:
        c = np.float32(self.params.cell_size)
        return (float(np.float32(self.width) * c), float(np.float32(self.height) * c),
                float(np.float32(self.depth) * c))

    def advance_clock(self, steps: int) -> None:
        """grid.step += n; grid.time += dt per step, in f32 (grid3d.rs:267-268)."""
        dt = np.float32(self.params.time_step)
        for _ in range(int(steps)):
            self.time = np.float32(self.time + dt)
        self.step += int(steps)

