"""B200-native WaveSim3D FDTD step (mivertowski/RustCompute ringkernel-wavesim3d).

Host-side mirror of the reference's simulation grid and GPU backend API over
libws3d.so, a hand-written sm_100a CUDA library with a plain C ABI
(include/ws3d.h).  There is no CPU fallback: every step runs on the GPU.
"""
from .grid import AcousticParams3D, CellType, SimulationGrid3D  # noqa: F401
from .backend import (  # noqa: F401
    CommandError, CompileError, DeviceError, GpuBackend3D, GpuError, InvalidArgument,
    LaunchError, MemoryError_, PeerError, ReadbackError, SimulationError, TimeoutError_,
)
from .persistent import (  # noqa: F401
    PersistentBackend, PersistentBackendConfig, PersistentBackendStats, ResponseType,
)
from . import configs  # noqa: F401

__all__ = [
    "AcousticParams3D", "CellType", "SimulationGrid3D", "GpuBackend3D", "GpuError",
    "DeviceError", "CompileError", "LaunchError", "MemoryError_", "SimulationError",
    "CommandError", "ReadbackError", "InvalidArgument", "TimeoutError_", "PeerError",
    "PersistentBackend", "PersistentBackendConfig", "PersistentBackendStats", "ResponseType",
    "configs",
]
