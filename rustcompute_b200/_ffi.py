"""ctypes binding of libws3d.so (the C-ABI declared in include/ws3d.h).

The library is loaded from the package directory only.  There is no fallback:
if the shared object is missing, importing the backend raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libws3d.so")

# ws3d_status values (include/ws3d.h)
WS3D_OK = 0
WS3D_EDEVICE = 1
WS3D_ECOMPILE = 2
WS3D_ELAUNCH = 3
WS3D_EMEMORY = 4
WS3D_ESIMULATION = 5
WS3D_ECOMMAND = 6
WS3D_EREADBACK = 7
WS3D_EINVAL = 8
WS3D_ETIMEOUT = 9
WS3D_EPEER = 10

WS3D_STATIC_ENERGY_MAX_PLANES = 8192   # include/ws3d.h
# rows of a two-step (k_step_tma2) tile, kTbTY in csrc/ws3d_index.h: the two-step
# kernel takes grids with W > 128 and H >= WS3D_TWO_STEP_ROWS + 4
WS3D_TWO_STEP_ROWS = 16

WS3D_VARIANT_AUTO = 0
WS3D_VARIANT_ZSTREAM = 1
WS3D_VARIANT_NAIVE = 2
WS3D_VARIANT_REFSHAPE = 3
WS3D_VARIANT_TMA = 4
WS3D_VARIANT_ASYNC = 5
WS3D_VARIANT_TMA2 = 6


class ws3d_desc(C.Structure):
    _fields_ = [
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("depth", C.c_uint32),
        ("c_squared", C.c_float),
        ("damping", C.c_float),
        ("sponge_width", C.c_uint32),
        ("sponge_max", C.c_float),
        ("device", C.c_int32),
        ("z_begin", C.c_uint32),
        ("z_end", C.c_uint32),
        ("variant", C.c_uint32),
        ("reserved0", C.c_uint32),
        ("spin_budget", C.c_uint64),
    ]


class ws3d_stats(C.Structure):
    _fields_ = [
        ("step", C.c_uint64),
        ("kernel_launches", C.c_uint64),
        ("device_bytes", C.c_uint64),
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("depth", C.c_uint32),
        ("z_begin", C.c_uint32),
        ("z_end", C.c_uint32),
        ("pitch", C.c_uint32),
        ("variant", C.c_uint32),
        ("has_c2_field", C.c_uint32),
        ("has_cell_field", C.c_uint32),
        ("n_sources", C.c_uint32),
        ("two_step_launches", C.c_uint32),
    ]


HALO_CAP_TWO_STEP = 1
HALO_CAP_C2_FIELD = 2


class ws3d_halo_handles(C.Structure):
    _fields_ = [
        ("buf", (C.c_uint8 * 64) * 4),
        ("flags", C.c_uint8 * 64),
        ("c2", C.c_uint8 * 64),
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("depth", C.c_uint32),
        ("pitch", C.c_uint32),
        ("z_begin", C.c_uint32),
        ("z_end", C.c_uint32),
        ("device", C.c_int32),
        ("caps", C.c_uint32),
        ("ghost_planes", C.c_uint32),
        ("c_squared", C.c_float),
    ]


# resident (command-driven) mode: message codes and layouts (include/ws3d.h)
WS3D_CMD_NOP = 0
WS3D_CMD_RUN_STEPS = 1
WS3D_CMD_PAUSE = 2
WS3D_CMD_RESUME = 3
WS3D_CMD_TERMINATE = 4
WS3D_CMD_INJECT_IMPULSE = 5
WS3D_CMD_SET_SOURCE = 6
WS3D_CMD_GET_PROGRESS = 7
WS3D_RESP_ACK = 0
WS3D_RESP_PROGRESS = 1
WS3D_RESP_ERROR = 2
WS3D_RESP_TERMINATED = 3
WS3D_RESP_ENERGY = 4


class ws3d_h2k_msg(C.Structure):
    _fields_ = [
        ("cmd", C.c_uint32),
        ("flags", C.c_uint32),
        ("cmd_id", C.c_uint64),
        ("param1", C.c_uint64),
        ("param2", C.c_uint32),
        ("param3", C.c_uint32),
        ("param4", C.c_float),
        ("param5", C.c_float),
        ("reserved", C.c_uint64 * 3),
    ]


class ws3d_k2h_msg(C.Structure):
    _fields_ = [
        ("resp_type", C.c_uint32),
        ("flags", C.c_uint32),
        ("cmd_id", C.c_uint64),
        ("step", C.c_uint64),
        ("steps_remaining", C.c_uint64),
        ("energy", C.c_float),
        ("error_code", C.c_uint32),
        ("reserved", C.c_uint64 * 3),
    ]


class ws3d_resident_config(C.Structure):
    _fields_ = [
        ("progress_interval", C.c_uint64),
        ("h2k_capacity", C.c_uint32),
        ("k2h_capacity", C.c_uint32),
        ("idle_budget_ns", C.c_uint64),
        ("reserved", C.c_uint64 * 4),
    ]


class ws3d_resident_stats(C.Structure):
    _fields_ = [
        ("current_step", C.c_uint64),
        ("steps_remaining", C.c_uint64),
        ("total_energy", C.c_float),
        ("has_terminated", C.c_uint32),
        ("messages_processed", C.c_uint64),
        ("k2h_dropped", C.c_uint64),
        ("launches", C.c_uint64),
        ("is_running", C.c_uint32),
        ("kernel_alive", C.c_uint32),
        ("paused", C.c_uint32),
        ("reserved32", C.c_uint32),
        ("reserved", C.c_uint64 * 3),
    ]


class ws3d_volume_params(C.Structure):
    _fields_ = [
        ("width", C.c_uint32),
        ("height", C.c_uint32),
        ("density_scale", C.c_float),
        ("step_size", C.c_float),
        ("max_steps", C.c_uint32),
        ("threshold", C.c_float),
        ("cell_size", C.c_float),
        ("fov_y", C.c_float),
        ("eye", C.c_float * 3),
        ("target", C.c_float * 3),
        ("up", C.c_float * 3),
        ("default_camera", C.c_uint32),
        ("background", C.c_float * 4),
        ("composite", C.c_uint32),
        ("reserved", C.c_uint32 * 3),
    ]


_P = C.c_void_p
_F = C.POINTER(C.c_float)
_U8 = C.POINTER(C.c_uint8)
_U32 = C.POINTER(C.c_uint32)
_CTX = C.c_void_p

# name -> (restype, argtypes).  Every symbol declared in include/ws3d.h.
SIGNATURES = {
    "ws3d_abi_version": (C.c_uint32, []),
    "ws3d_status_string": (C.c_char_p, [C.c_int]),
    "ws3d_desc_init": (None, [C.POINTER(ws3d_desc), C.c_uint32, C.c_uint32, C.c_uint32]),
    "ws3d_create": (C.c_int, [C.POINTER(ws3d_desc), C.POINTER(_CTX)]),
    "ws3d_destroy": (None, [_CTX]),
    "ws3d_last_error": (C.c_char_p, [_CTX]),
    "ws3d_upload": (C.c_int, [_CTX, _F, _F]),
    "ws3d_download": (C.c_int, [_CTX, _F, _F]),
    "ws3d_reset": (C.c_int, [_CTX, _F, _F]),
    "ws3d_set_step": (C.c_int, [_CTX, C.c_uint64]),
    "ws3d_set_cells": (C.c_int, [_CTX, _U8, _F]),
    "ws3d_set_c2_field": (C.c_int, [_CTX, _F]),
    "ws3d_set_sources": (C.c_int, [_CTX, C.c_uint32, _U32, _F, C.c_uint64]),
    "ws3d_step": (C.c_int, [_CTX, C.c_uint64]),
    "ws3d_step_timed": (C.c_int, [_CTX, C.c_uint64, C.POINTER(C.c_double)]),
    "ws3d_step_timed_begin": (C.c_int, [_CTX, C.c_uint64]),
    "ws3d_step_timed_end": (C.c_int, [_CTX, C.POINTER(C.c_double)]),
    "ws3d_halo_wait_stats": (C.c_int, [_CTX, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                       C.c_int]),
    "ws3d_step_persistent": (C.c_int, [_CTX, C.c_uint64]),
    "ws3d_inject_impulse": (C.c_int, [_CTX, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]),
    "ws3d_inject_spherical_impulse": (
        C.c_int, [_CTX, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float, C.c_float]),
    "ws3d_energy": (C.c_int, [_CTX, C.POINTER(C.c_double)]),
    "ws3d_max_pressure": (C.c_int, [_CTX, _F]),
    "ws3d_field_energy_static": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                           _P, _P, C.c_char_p, C.c_size_t]),
    "ws3d_memory_usage": (C.c_size_t, [_CTX]),
    "ws3d_get_slice": (C.c_int, [_CTX, C.c_uint32, C.c_uint32, _F]),
    "ws3d_sample_pressure": (C.c_int, [_CTX, C.c_uint32, _F, C.c_float, _F]),
    "ws3d_sync": (C.c_int, [_CTX]),
    "ws3d_set_stream": (C.c_int, [_CTX, _P]),
    "ws3d_get_stream": (C.c_int, [_CTX, C.POINTER(_P)]),
    "ws3d_stats_get": (C.c_int, [_CTX, C.POINTER(ws3d_stats)]),
    "ws3d_halo_export": (C.c_int, [_CTX, C.POINTER(ws3d_halo_handles)]),
    "ws3d_halo_attach": (C.c_int, [_CTX, C.POINTER(ws3d_halo_handles),
                                   C.POINTER(ws3d_halo_handles)]),
    "ws3d_halo_attach_local": (C.c_int, [_CTX, _CTX, _CTX]),
    "ws3d_halo_sync": (C.c_int, [_CTX, C.c_uint32]),
    "ws3d_halo_set_depth": (C.c_int, [_CTX, C.c_uint32]),
    "ws3d_step_group": (C.c_int, [C.POINTER(_CTX), C.c_uint32, C.c_uint64]),
    "ws3d_resident_start": (C.c_int, [_CTX, C.POINTER(ws3d_resident_config)]),
    "ws3d_resident_send": (C.c_int, [_CTX, C.POINTER(ws3d_h2k_msg)]),
    "ws3d_resident_run_steps": (C.c_int, [_CTX, C.c_uint64]),
    "ws3d_resident_inject_impulse": (
        C.c_int, [_CTX, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]),
    "ws3d_resident_wait_step": (C.c_int, [_CTX, C.c_uint64, C.c_uint64]),
    "ws3d_resident_poll": (C.c_int, [_CTX, C.POINTER(ws3d_k2h_msg), C.c_uint32, _U32]),
    "ws3d_resident_stats_get": (C.c_int, [_CTX, C.POINTER(ws3d_resident_stats)]),
    "ws3d_resident_download": (C.c_int, [_CTX, _F, C.c_uint64]),
    "ws3d_resident_shutdown": (C.c_int, [_CTX, C.c_uint64]),
    "ws3d_volume_params_init": (None, [C.POINTER(ws3d_volume_params), C.c_uint32, C.c_uint32]),
    "ws3d_render_volume": (C.c_int, [_CTX, C.POINTER(ws3d_volume_params), _F]),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load libws3d.so and bind every declared symbol (raises if absent)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            raise ImportError(
                f"{_LIB_PATH} is missing: build it with `python -m rustcompute_b200.build` "
                "(there is no CPU fallback)")
        lib = C.CDLL(_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib
