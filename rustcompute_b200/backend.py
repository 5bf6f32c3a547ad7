"""GpuBackend3D: the drop-in GPU backend over libws3d.so.

Mirrors crates/ringkernel-wavesim3d/src/simulation/gpu_backend.rs:172-494
(same method names, argument meaning and error behaviour): `step` advances
grid.step / grid.time but leaves grid.pressure alone until
`download_pressure`, exactly like gpu_backend.rs:314-380.  Errors are raised
as GpuError subclasses (gpu_backend.rs:13-23) and are never swallowed: there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _ffi
from .grid import SimulationGrid3D


class GpuError(RuntimeError):
    """gpu_backend.rs:13-23."""

    status = -1


class DeviceError(GpuError):
    status = _ffi.WS3D_EDEVICE


class CompileError(GpuError):
    status = _ffi.WS3D_ECOMPILE


class LaunchError(GpuError):
    status = _ffi.WS3D_ELAUNCH


class MemoryError_(GpuError):
    status = _ffi.WS3D_EMEMORY


class SimulationError(GpuError):
    status = _ffi.WS3D_ESIMULATION


class CommandError(GpuError):
    status = _ffi.WS3D_ECOMMAND


class ReadbackError(GpuError):
    status = _ffi.WS3D_EREADBACK


class InvalidArgument(GpuError):
    status = _ffi.WS3D_EINVAL


class TimeoutError_(GpuError):
    status = _ffi.WS3D_ETIMEOUT


class PeerError(GpuError):
    status = _ffi.WS3D_EPEER


_BY_STATUS = {cls.status: cls for cls in (
    DeviceError, CompileError, LaunchError, MemoryError_, SimulationError, CommandError,
    ReadbackError, InvalidArgument, TimeoutError_, PeerError)}


def _raise(lib, status: int, ctx, what: str) -> None:
    if status == _ffi.WS3D_OK:
        return
    msg = lib.ws3d_status_string(status).decode()
    detail = lib.ws3d_last_error(ctx).decode() if ctx else ""
    cls = _BY_STATUS.get(status, GpuError)
    raise cls(f"{what}: {msg}" + (f": {detail}" if detail else ""))


def _fptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _f32c(a, n: int, name: str) -> np.ndarray:
    arr = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    if arr.size != n:
        raise InvalidArgument(f"{name}: expected {n} values, got {arr.size}")
    return arr


VARIANTS = {"auto": _ffi.WS3D_VARIANT_AUTO, "zstream": _ffi.WS3D_VARIANT_ZSTREAM,
            "naive": _ffi.WS3D_VARIANT_NAIVE, "refshape": _ffi.WS3D_VARIANT_REFSHAPE,
            "tma": _ffi.WS3D_VARIANT_TMA, "async": _ffi.WS3D_VARIANT_ASYNC,
            "tma2": _ffi.WS3D_VARIANT_TMA2}


class GpuBackend3D:
    """GPU backend for one grid, or for one z-slab [z_begin, z_end) of it."""

    def __init__(self, grid: SimulationGrid3D, *, device: int = 0, variant: str = "auto",
                 sponge_width: int = 0, sponge_max: float = 0.0,
                 z_begin: int = 0, z_end: int = 0, upload: bool = True):
        """GpuBackend3D::new (gpu_backend.rs:204-311): device state for `grid`
        (or for its planes [z_begin, z_end)), then upload of its fields and,
        when they differ from the default face layout, its cell arrays."""
        self._open(grid.width, grid.height, grid.depth, grid.params.c_squared,
                   grid.params.simple_damping, device=device, variant=variant,
                   sponge_width=sponge_width, sponge_max=sponge_max, z_begin=z_begin,
                   z_end=z_end)
        if upload:
            if not grid.has_default_cells():
                self.set_cells(grid.cell_types, grid.reflection_coeff)
            self.upload_pressure(grid)

    @classmethod
    def create(cls, width: int, height: int, depth: int, *, c_squared: float = 0.25,
               damping: float = 1.0, device: int = 0, variant: str = "auto",
               sponge_width: int = 0, sponge_max: float = 0.0, z_begin: int = 0,
               z_end: int = 0, spin_budget_ns: int = 0) -> "GpuBackend3D":
        """A backend without a host grid (fields start at zero).  z_begin/z_end
        select a z-slab; spin_budget_ns bounds the device-side halo waits
        (0 = library default, 2 s)."""
        self = cls.__new__(cls)
        self._open(width, height, depth, c_squared, damping, device=device, variant=variant,
                   sponge_width=sponge_width, sponge_max=sponge_max, z_begin=z_begin,
                   z_end=z_end, spin_budget_ns=spin_budget_ns)
        return self

    def _open(self, width, height, depth, c_squared, damping, *, device, variant,
              sponge_width, sponge_max, z_begin, z_end, spin_budget_ns=0):
        self._ctx = None
        self._lib = _ffi.load()
        d = _ffi.ws3d_desc()
        self._lib.ws3d_desc_init(C.byref(d), width, height, depth)
        d.c_squared = np.float32(c_squared)
        d.damping = np.float32(damping)
        d.sponge_width = int(sponge_width)
        d.sponge_max = np.float32(sponge_max)
        d.device = int(device)
        d.z_begin, d.z_end = int(z_begin), int(z_end)
        d.spin_budget = int(spin_budget_ns)
        if variant not in VARIANTS:
            raise InvalidArgument(f"unknown variant {variant!r}; one of {sorted(VARIANTS)}")
        d.variant = VARIANTS[variant]
        ctx = C.c_void_p()
        st = self._lib.ws3d_create(C.byref(d), C.byref(ctx))
        if st != _ffi.WS3D_OK:
            _raise(self._lib, st, None, "GpuBackend3D::new")
        self._ctx = ctx
        self.width, self.height, self.depth = int(width), int(height), int(depth)
        self.z_begin = int(z_begin)
        self.z_end = int(z_end) if z_end else self.depth
        ss = self.width * self.height
        self._slab = slice(self.z_begin * ss, self.z_end * ss)
        self.n_local = (self.z_end - self.z_begin) * ss

    # -- lifetime ---------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            self._lib.ws3d_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _chk(self, st: int, what: str) -> None:
        if st != _ffi.WS3D_OK:
            _raise(self._lib, st, self._ctx, what)

    # -- reference API (gpu_backend.rs) ----------------------------------------
    def step(self, grid: Optional[SimulationGrid3D] = None) -> None:
        """One FDTD step (gpu_backend.rs:314-380); asynchronous."""
        self._chk(self._lib.ws3d_step(self._ctx, 1), "GpuBackend3D::step")
        if grid is not None:
            grid.advance_clock(1)

    def step_n(self, grid: Optional[SimulationGrid3D], n: int) -> None:
        """`n` steps in one call (SimulationEngine::step_n, mod.rs:304)."""
        self._chk(self._lib.ws3d_step(self._ctx, int(n)), "GpuBackend3D::step_n")
        if grid is not None:
            grid.advance_clock(n)

    def step_persistent(self, n: int) -> None:
        """`n` steps in one cooperative launch (bit-identical to step_n)."""
        self._chk(self._lib.ws3d_step_persistent(self._ctx, int(n)), "step_persistent")

    def step_timed(self, n: int) -> float:
        """`n` steps; returns the summed device time of the step-kernel launches
        in ms (CUDA events on the launch stream).  Synchronises."""
        out = C.c_double()
        self._chk(self._lib.ws3d_step_timed(self._ctx, int(n), C.byref(out)), "step_timed")
        return float(out.value)

    def step_timed_begin(self, n: int) -> None:
        """step_timed without the synchronisation: enqueues `n` timed steps, so
        the caller can record its own event right behind the last launch."""
        self._chk(self._lib.ws3d_step_timed_begin(self._ctx, int(n)), "step_timed_begin")

    def step_timed_end(self) -> float:
        """Synchronises and returns the summed kernel time (ms) of the launches
        since step_timed_begin."""
        out = C.c_double()
        self._chk(self._lib.ws3d_step_timed_end(self._ctx, C.byref(out)), "step_timed_end")
        return float(out.value)

    def halo_wait_stats(self, reset: bool = False) -> tuple[int, int]:
        """z-slabs: (device ns spent in neighbour-flag waits that did not pass at
        once, number of such waits) since the last reset.  Synchronises."""
        ns, cnt = C.c_uint64(), C.c_uint64()
        self._chk(self._lib.ws3d_halo_wait_stats(self._ctx, C.byref(ns), C.byref(cnt),
                                                 1 if reset else 0), "halo_wait_stats")
        return int(ns.value), int(cnt.value)

    def download_pressure(self, grid: SimulationGrid3D, with_prev: bool = False) -> None:
        """gpu_backend.rs:383-388 (synchronous)."""
        p = np.empty(self.n_local, dtype=np.float32)
        pp = np.empty(self.n_local, dtype=np.float32) if with_prev else None
        self._chk(self._lib.ws3d_download(self._ctx, _fptr(p), _fptr(pp)),
                  "GpuBackend3D::download_pressure")
        grid.pressure[self._slab] = p
        if pp is not None:
            grid.pressure_prev[self._slab] = pp

    def upload_pressure(self, grid: SimulationGrid3D) -> None:
        """gpu_backend.rs:391-401."""
        p = _f32c(grid.pressure[self._slab], self.n_local, "pressure")
        pp = _f32c(grid.pressure_prev[self._slab], self.n_local, "pressure_prev")
        self._chk(self._lib.ws3d_upload(self._ctx, _fptr(p), _fptr(pp)),
                  "GpuBackend3D::upload_pressure")

    def reset(self, grid: SimulationGrid3D) -> None:
        """gpu_backend.rs:404-408."""
        p = _f32c(grid.pressure[self._slab], self.n_local, "pressure")
        pp = _f32c(grid.pressure_prev[self._slab], self.n_local, "pressure_prev")
        self._chk(self._lib.ws3d_reset(self._ctx, _fptr(p), _fptr(pp)), "GpuBackend3D::reset")

    def inject_impulse(self, x: int, y: int, z: int, amplitude: float) -> None:
        """gpu_backend.rs:411-442."""
        self._chk(self._lib.ws3d_inject_impulse(self._ctx, x, y, z, np.float32(amplitude)),
                  "GpuBackend3D::inject_impulse")

    def inject_spherical_impulse(self, cx: int, cy: int, cz: int, amplitude: float,
                                 radius: float) -> None:
        """gpu_backend.rs:445-487 with the CPU factor exp(-d2/(2r))."""
        self._chk(self._lib.ws3d_inject_spherical_impulse(
            self._ctx, cx, cy, cz, np.float32(amplitude), np.float32(radius)),
            "GpuBackend3D::inject_spherical_impulse")

    def get_xy_slice(self, z: int) -> np.ndarray:
        """grid3d.rs:414-418, read from the device."""
        out = np.empty(self.width * self.height, np.float32)
        self._chk(self._lib.ws3d_get_slice(self._ctx, 0, int(z), _fptr(out)), "get_xy_slice")
        return out

    def get_xz_slice(self, y: int) -> np.ndarray:
        """grid3d.rs:421-430 (owned planes), read from the device."""
        out = np.empty(self.width * (self.z_end - self.z_begin), np.float32)
        self._chk(self._lib.ws3d_get_slice(self._ctx, 1, int(y), _fptr(out)), "get_xz_slice")
        return out

    def get_yz_slice(self, x: int) -> np.ndarray:
        """grid3d.rs:433-442 (owned planes), read from the device."""
        out = np.empty(self.height * (self.z_end - self.z_begin), np.float32)
        self._chk(self._lib.ws3d_get_slice(self._ctx, 2, int(x), _fptr(out)), "get_yz_slice")
        return out

    def sample_pressure(self, positions_m, cell_size: float) -> np.ndarray:
        """grid3d.rs:373-411 at (n, 3) positions in metres; f32 samples."""
        pos = np.ascontiguousarray(positions_m, dtype=np.float32).reshape(-1, 3)
        out = np.empty(pos.shape[0], np.float32)
        self._chk(self._lib.ws3d_sample_pressure(self._ctx, pos.shape[0], _fptr(pos),
                                                 np.float32(cell_size), _fptr(out)),
                  "sample_pressure")
        return out

    def memory_usage(self) -> int:
        """gpu_backend.rs:490-493 (actual device bytes held)."""
        return int(self._lib.ws3d_memory_usage(self._ctx))

    # -- north-star extensions ---------------------------------------------------
    def set_cells(self, cell_types: np.ndarray, reflection: np.ndarray) -> None:
        t = np.ascontiguousarray(cell_types, dtype=np.uint8).reshape(-1)
        r = np.ascontiguousarray(reflection, dtype=np.float32).reshape(-1)
        if t.size == self.width * self.height * self.depth and t.size != self.n_local:
            t, r = t[self._slab].copy(), r[self._slab].copy()
        if t.size != self.n_local or r.size != self.n_local:
            raise InvalidArgument("set_cells: array size does not match the grid")
        self._chk(self._lib.ws3d_set_cells(self._ctx, t.ctypes.data_as(C.POINTER(C.c_uint8)),
                                           _fptr(r)), "set_cells")

    def set_c2_field(self, c2: Optional[np.ndarray]) -> None:
        if c2 is None:
            self._chk(self._lib.ws3d_set_c2_field(self._ctx, None), "set_c2_field")
            return
        a = np.ascontiguousarray(c2, dtype=np.float32).reshape(-1)
        if a.size == self.width * self.height * self.depth and a.size != self.n_local:
            a = a[self._slab].copy()
        a = _f32c(a, self.n_local, "c2")
        self._chk(self._lib.ws3d_set_c2_field(self._ctx, _fptr(a)), "set_c2_field")

    def set_sources(self, xyz: np.ndarray, wavelet: np.ndarray) -> None:
        """Point sources (global x,y,z) driven by per-source wavelets
        (shape [n, len]) with the inject_impulse semantic before each step."""
        xyz = np.ascontiguousarray(xyz, dtype=np.uint32).reshape(-1, 3)
        wl = np.ascontiguousarray(wavelet, dtype=np.float32)
        n = xyz.shape[0]
        if n == 0:
            self._chk(self._lib.ws3d_set_sources(self._ctx, 0, None, None, 0), "set_sources")
            return
        wl = wl.reshape(n, -1)
        self._chk(self._lib.ws3d_set_sources(
            self._ctx, n, xyz.ctypes.data_as(C.POINTER(C.c_uint32)), _fptr(wl), wl.shape[1]),
            "set_sources")

    def energy(self) -> float:
        out = C.c_double()
        self._chk(self._lib.ws3d_energy(self._ctx, C.byref(out)), "energy")
        return float(out.value)

    def max_pressure(self) -> float:
        out = C.c_float()
        self._chk(self._lib.ws3d_max_pressure(self._ctx, C.byref(out)), "max_pressure")
        return float(out.value)

    def sync(self) -> None:
        self._chk(self._lib.ws3d_sync(self._ctx), "sync")

    def set_stream(self, stream_handle: int | None) -> None:
        self._chk(self._lib.ws3d_set_stream(self._ctx, C.c_void_p(stream_handle or 0)),
                  "set_stream")

    def stream_handle(self) -> int:
        out = C.c_void_p()
        self._chk(self._lib.ws3d_get_stream(self._ctx, C.byref(out)), "get_stream")
        return int(out.value or 0)

    def volume_params(self, width: int = 640, height: int = 360, *, density_scale: float = 2.0,
                      step_size: float = 0.05, max_steps: int = 256, threshold: float = 0.01,
                      cell_size: float = 1.0, fov_y: Optional[float] = None, eye=None,
                      target=None, up=(0.0, 1.0, 0.0), background=None):
        """VolumeParams (volume.rs:166-190) plus the camera (camera.rs): the
        default camera is Camera3D::for_grid; `background` (RGBA) turns on
        ALPHA_BLENDING compositing."""
        prm = _ffi.ws3d_volume_params()
        self._lib.ws3d_volume_params_init(C.byref(prm), int(width), int(height))
        prm.density_scale = density_scale
        prm.step_size = step_size
        prm.max_steps = int(max_steps)
        prm.threshold = threshold
        prm.cell_size = cell_size
        if fov_y is not None:
            prm.fov_y = fov_y
        if eye is not None:
            prm.default_camera = 0
            prm.eye[:] = [float(v) for v in eye]
            prm.target[:] = [float(v) for v in target]
        prm.up[:] = [float(v) for v in up]
        if background is not None:
            prm.composite = 1
            prm.background[:] = [float(v) for v in background]
        return prm

    def render_volume(self, width: int = 640, height: int = 360, **kw) -> np.ndarray:
        """Headless volume ray-march of the current pressure (volume.rs:76-160):
        float32 RGBA image of shape (height, width, 4), row 0 at the top."""
        prm = self.volume_params(width, height, **kw)
        out = np.empty((int(height), int(width), 4), dtype=np.float32)
        self._chk(self._lib.ws3d_render_volume(self._ctx, C.byref(prm), _fptr(out)),
                  "render_volume")
        return out

    def stats(self) -> dict:
        s = _ffi.ws3d_stats()
        self._chk(self._lib.ws3d_stats_get(self._ctx, C.byref(s)), "stats")
        return {name: getattr(s, name) for name, _ in s._fields_ if name != "reserved"}

    def upload_fields(self, p: np.ndarray, pp: Optional[np.ndarray] = None) -> None:
        """Upload the owned planes from flat f32 arrays (pinned or pageable)."""
        p = _f32c(p, self.n_local, "pressure")
        pp = None if pp is None else _f32c(pp, self.n_local, "pressure_prev")
        self._chk(self._lib.ws3d_upload(self._ctx, _fptr(p), _fptr(pp)), "upload")

    def download_into(self, p: np.ndarray, pp: Optional[np.ndarray] = None) -> None:
        """Download the owned planes into caller-provided flat f32 arrays."""
        for a in (p, pp):
            if a is not None and (a.dtype != np.float32 or a.size != self.n_local
                                  or not a.flags.c_contiguous):
                raise InvalidArgument("download_into: need contiguous f32 of the slab size")
        self._chk(self._lib.ws3d_download(self._ctx, _fptr(p), _fptr(pp)), "download")

    def download_field(self, with_prev: bool = False):
        p = np.empty(self.n_local, dtype=np.float32)
        pp = np.empty(self.n_local, dtype=np.float32) if with_prev else None
        self._chk(self._lib.ws3d_download(self._ctx, _fptr(p), _fptr(pp)), "download")
        return (p, pp) if with_prev else p
