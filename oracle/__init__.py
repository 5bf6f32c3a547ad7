"""CPU oracle for the WaveSim3D FDTD step -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py may
import this package.  It wraps oracle/_build/libws3d_oracle.so, a C
restatement of crates/ringkernel-wavesim3d/src/simulation/grid3d.rs
(step_sequential :222-269, step_parallel :272-350, boundaries :353-370,
injection :146-191), compiled with -ffp-contract=off.

Parity status: the reference (Rust, wgpu-dependent) cannot be built in this
image.  The restatement is pinned by the reference's own known-answer tests
(restated in tests/test_oracle.py) and by an analytic eigenmode solution of
the discrete scheme; no field dump made by the reference itself exists.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

from rustcompute_b200.grid import SimulationGrid3D

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "libws3d_oracle.so")


def build() -> str:
    src = os.path.join(HERE, "ws3d_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


class _Params(C.Structure):
    _fields_ = [("c_squared", C.c_float), ("damping", C.c_float),
                ("c2_field", C.c_void_p), ("sponge", C.c_void_p), ("sponge_w", C.c_uint32)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        u32, f32, vp = C.c_uint32, C.c_float, C.c_void_p
        L.ws3o_setup_boundaries.argtypes = [u32, u32, u32, vp, vp]
        L.ws3o_inject_impulse.argtypes = [u32, u32, u32, vp, vp, u32, u32, u32, f32]
        L.ws3o_inject_spherical.argtypes = [u32, u32, u32, vp, vp, u32, u32, u32, f32, f32]
        L.ws3o_sponge_table.argtypes = [u32, f32, vp]
        L.ws3o_step_sequential.argtypes = [u32, u32, u32, vp, vp, vp, vp, C.POINTER(_Params)]
        L.ws3o_step_parallel.argtypes = [u32, u32, u32, vp, vp, vp, vp, C.POINTER(_Params), C.c_int]
        L.ws3o_run.argtypes = [u32, u32, u32, vp, vp, vp, vp, C.POINTER(_Params), C.c_uint64,
                               C.c_uint64, u32, vp, vp, C.c_uint64, C.c_int]
        L.ws3o_run_swap.argtypes = L.ws3o_run.argtypes
        L.ws3o_run_swap.restype = C.c_int
        L.ws3o_total_energy_f32.argtypes = [vp, C.c_uint64]
        L.ws3o_total_energy_f32.restype = f32
        L.ws3o_total_energy_f64.argtypes = [vp, C.c_uint64]
        L.ws3o_total_energy_f64.restype = C.c_double
        L.ws3o_max_pressure.argtypes = [vp, C.c_uint64]
        L.ws3o_max_pressure.restype = f32
        L.ws3o_max_threads.restype = C.c_int
        L.ws3o_render_volume.argtypes = [vp, u32, u32, u32, vp, vp]
        L.ws3o_render_volume.restype = C.c_int
        L.ws3o_quantize_f16.argtypes = [vp, C.c_uint64, vp]
        _lib = L
    return _lib


class _VolumeParams(C.Structure):
    """Layout of ws3o_volume_params (the same fields as ws3d_volume_params)."""
    _fields_ = [
        ("width", C.c_uint32), ("height", C.c_uint32), ("density_scale", C.c_float),
        ("step_size", C.c_float), ("max_steps", C.c_uint32), ("threshold", C.c_float),
        ("cell_size", C.c_float), ("fov_y", C.c_float), ("eye", C.c_float * 3),
        ("target", C.c_float * 3), ("up", C.c_float * 3), ("default_camera", C.c_uint32),
        ("background", C.c_float * 4), ("composite", C.c_uint32), ("reserved", C.c_uint32 * 3),
    ]


def render_volume(p: np.ndarray, W: int, H: int, D: int, width: int = 640, height: int = 360, *,
                  density_scale: float = 2.0, step_size: float = 0.05, max_steps: int = 256,
                  threshold: float = 0.01, cell_size: float = 1.0, fov_y: float = None, eye=None,
                  target=None, up=(0.0, 1.0, 0.0), background=None) -> np.ndarray:
    """CPU restatement of the volume ray-march (visualization/volume.rs:76-160,
    :396-420; camera.rs:51-61): float32 RGBA image (height, width, 4)."""
    prm = _VolumeParams(width=int(width), height=int(height), density_scale=density_scale,
                        step_size=step_size, max_steps=int(max_steps), threshold=threshold,
                        cell_size=cell_size,
                        fov_y=np.float32(0.785398163397448309616) if fov_y is None else fov_y)
    prm.default_camera = 1 if eye is None else 0
    if eye is not None:
        prm.eye[:] = [float(v) for v in eye]
        prm.target[:] = [float(v) for v in target]
    prm.up[:] = [float(v) for v in up]
    if background is not None:
        prm.composite = 1
        prm.background[:] = [float(v) for v in background]
    f = np.ascontiguousarray(p, dtype=np.float32).reshape(-1)
    assert f.size == W * H * D
    out = np.empty((int(height), int(width), 4), dtype=np.float32)
    if lib().ws3o_render_volume(f.ctypes.data_as(C.c_void_p), W, H, D, C.byref(prm),
                                out.ctypes.data_as(C.c_void_p)) != 0:
        raise ValueError("render_volume: degenerate camera")
    return out


def quantize_f16(x: np.ndarray) -> np.ndarray:
    """The renderer's f32 -> f16 (round to nearest even) -> f32."""
    f = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty_like(f)
    lib().ws3o_quantize_f16(f.ctypes.data_as(C.c_void_p), f.size, out.ctypes.data_as(C.c_void_p))
    return out


def _ptr(a):
    return None if a is None else a.ctypes.data


def sponge_table(width: int, smax: float) -> np.ndarray:
    out = np.zeros(max(width, 1), dtype=np.float32)
    if width:
        lib().ws3o_sponge_table(width, np.float32(smax), _ptr(out))
    return out[:width]


def max_threads() -> int:
    return int(lib().ws3o_max_threads())


class OracleGrid(SimulationGrid3D):
    """SimulationGrid3D plus the reference CPU steps (grid3d.rs:222-350).

    Extensions (all off by default): c2_field (per-cell Courant^2), sponge
    (width, smax), point sources driven with the inject_impulse semantic.
    """

    def __init__(self, width, height, depth, params=None, *, c2_field=None,
                 sponge_width=0, sponge_max=0.0):
        super().__init__(width, height, depth, params)
        self.c2_field = None if c2_field is None else np.ascontiguousarray(c2_field, np.float32).reshape(-1)
        self.sponge_width = int(sponge_width)
        self._sponge = sponge_table(self.sponge_width, sponge_max) if sponge_width else None
        self.src_idx = np.zeros(0, dtype=np.uint64)
        self.wavelet = np.zeros((0, 1), dtype=np.float32)
        self.use_cells = False  # False: default face layout evaluated analytically

    def set_cell_type(self, x, y, z, cell_type):
        super().set_cell_type(x, y, z, cell_type)
        self.use_cells = True

    def set_sources(self, xyz, wavelet):
        xyz = np.asarray(xyz, dtype=np.int64).reshape(-1, 3)
        self.src_idx = np.array([self.index(int(x), int(y), int(z)) for x, y, z in xyz],
                                dtype=np.uint64)
        self.wavelet = np.ascontiguousarray(wavelet, dtype=np.float32).reshape(len(xyz), -1) \
            if len(xyz) else np.zeros((0, 1), dtype=np.float32)

    def _params(self):
        return _Params(np.float32(self.params.c_squared), np.float32(self.params.simple_damping),
                       _ptr(self.c2_field), _ptr(self._sponge), self.sponge_width)

    def _cells(self):
        if self.use_cells:
            return _ptr(self.cell_types), _ptr(self.reflection_coeff)
        return None, None

    def step_sequential(self):
        t, r = self._cells()
        prm = self._params()
        lib().ws3o_step_sequential(self.width, self.height, self.depth, _ptr(self.pressure),
                                   _ptr(self.pressure_prev), t, r, C.byref(prm))
        self.pressure, self.pressure_prev = self.pressure_prev, self.pressure
        self.advance_clock(1)

    def step_parallel(self, nthreads: int = 0):
        t, r = self._cells()
        prm = self._params()
        lib().ws3o_step_parallel(self.width, self.height, self.depth, _ptr(self.pressure),
                                 _ptr(self.pressure_prev), t, r, C.byref(prm),
                                 nthreads or max_threads())
        self.pressure, self.pressure_prev = self.pressure_prev, self.pressure
        self.advance_clock(1)

    def run(self, nsteps: int, nthreads: int = 1):
        """nsteps steps (sources applied before each); nthreads > 1 uses the
        parallel restatement.  Keeps self.pressure / pressure_prev roles."""
        t, r = self._cells()
        prm = self._params()
        n_src = len(self.src_idx)
        wl_len = self.wavelet.shape[1] if n_src else 0
        swapped = lib().ws3o_run_swap(self.width, self.height, self.depth, _ptr(self.pressure),
                                      _ptr(self.pressure_prev), t, r, C.byref(prm), self.step,
                                      nsteps, n_src, _ptr(self.src_idx) if n_src else None,
                                      _ptr(self.wavelet) if n_src else None, wl_len,
                                      int(nthreads))
        if swapped:
            self.pressure, self.pressure_prev = self.pressure_prev, self.pressure
        self.advance_clock(nsteps)

    def inject_spherical_impulse(self, cx, cy, cz, amplitude, radius):
        lib().ws3o_inject_spherical(self.width, self.height, self.depth, _ptr(self.pressure),
                                    _ptr(self.pressure_prev), cx, cy, cz, np.float32(amplitude),
                                    np.float32(radius))

    def inject_impulse_c(self, x, y, z, amplitude):
        lib().ws3o_inject_impulse(self.width, self.height, self.depth, _ptr(self.pressure),
                                  _ptr(self.pressure_prev), x, y, z, np.float32(amplitude))

    def total_energy_f32(self) -> float:
        return float(lib().ws3o_total_energy_f32(_ptr(self.pressure), self.total_cells))


def from_workload(wl, steps=None, z_begin=0, z_end=None) -> OracleGrid:
    """Oracle grid initialised with a configs.Workload's inputs."""
    from rustcompute_b200.grid import AcousticParams3D
    prm = AcousticParams3D(c_squared=wl.c_squared, simple_damping=wl.damping)
    g = OracleGrid(wl.W, wl.H, wl.D, prm, c2_field=wl.c2_field(),
                   sponge_width=wl.sponge_width, sponge_max=wl.sponge_max)
    p, pp = wl.initial_fields()
    g.pressure[:] = p
    g.pressure_prev[:] = pp
    if len(wl.sources):
        g.set_sources(wl.sources, wl.wavelet)
    return g
