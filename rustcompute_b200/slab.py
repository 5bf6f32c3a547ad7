"""z-slab decomposition of the grid over GPUs (host side).

One process per GPU (torchrun): rank r owns planes slab_bounds(D, world, r).
The ranks exchange the IPC handles of their field buffers and flag blocks
with one all_gather over torch.distributed (host plumbing only); from then on
the halo moves inside the step kernel over NVLink (include/ws3d.h, section
"z-slab decomposition").

Temporal depth 2 (two steps per exchange, two ghost planes per side) is
taken when every rank's export says it can: the choice must be the same on
all ranks, so it is made from the gathered handles, not per rank.

LocalSlabGroup runs the same decomposition inside one process on one GPU
(stream-ordered, no device waits); it exists to test the slab arithmetic on a
single device.
"""
from __future__ import annotations

import ctypes as C
import time
from typing import Callable, Optional, Sequence

from . import _ffi
from .backend import GpuBackend3D


def slab_bounds(D: int, world: int, rank: int) -> tuple[int, int]:
    """Planes [z_begin, z_end) of `rank`: D split as evenly as possible."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if D < world:
        raise ValueError(f"depth {D} is smaller than the number of slabs {world}")
    base, extra = divmod(D, world)
    zb = rank * base + min(rank, extra)
    return zb, zb + base + (1 if rank < extra else 0)


def neighbours(rank: int, world: int) -> tuple[Optional[int], Optional[int]]:
    return (rank - 1 if rank > 0 else None), (rank + 1 if rank + 1 < world else None)


def export_handles(b: GpuBackend3D) -> bytes:
    h = _ffi.ws3d_halo_handles()
    b._chk(b._lib.ws3d_halo_export(b._ctx, C.byref(h)), "halo_export")
    return bytes(h)


def _handles(blob: Optional[bytes]):
    if blob is None:
        return None
    h = _ffi.ws3d_halo_handles()
    C.memmove(C.byref(h), blob, C.sizeof(h))
    return h


def attach(b: GpuBackend3D, lower: Optional[bytes], upper: Optional[bytes]) -> None:
    lo, hi = _handles(lower), _handles(upper)
    b._chk(b._lib.ws3d_halo_attach(b._ctx, C.byref(lo) if lo else None,
                                   C.byref(hi) if hi else None), "halo_attach")


def temporal_depth(blobs: Sequence[bytes]) -> int:
    """Steps per exchange all ranks can take: 2 when every slab is two-step
    capable, owns >= 2 planes, and c2 is given the same way on all of them
    (a field everywhere, or one uniform value), else 1."""
    hs = [_handles(x) for x in blobs]
    if len(hs) < 2:
        return 1
    two = all(h.caps & _ffi.HALO_CAP_TWO_STEP and h.z_end - h.z_begin >= 2 for h in hs)
    fields = {bool(h.caps & _ffi.HALO_CAP_C2_FIELD) for h in hs}
    uniform = {h.c_squared for h in hs}
    same_c2 = fields == {True} or (fields == {False} and len(uniform) == 1)
    return 2 if two and same_c2 else 1


def set_depth(b: GpuBackend3D, depth: int) -> None:
    b._chk(b._lib.ws3d_halo_set_depth(b._ctx, int(depth)), "halo_set_depth")


def halo_sync(b: GpuBackend3D, barrier: Callable[[], None]) -> None:
    """Collective: clear flags, barrier, push boundary planes, barrier."""
    b._chk(b._lib.ws3d_halo_sync(b._ctx, 0), "halo_sync(0)")
    barrier()
    b._chk(b._lib.ws3d_halo_sync(b._ctx, 1), "halo_sync(1)")
    barrier()


def gather_handles(blob: bytes, rank: int, world: int, all_gather_object) -> list:
    """All ranks' handle blobs, in rank order (all_gather_object semantics)."""
    out = [None] * world
    all_gather_object(out, blob)
    return out


def connect(b: GpuBackend3D, rank: int, world: int, all_gather_object,
            barrier: Callable[[], None], depth: Optional[int] = None,
            timings: Optional[dict] = None) -> int:
    """Exchange handles, attach both neighbours, pick the temporal depth
    (`depth`, or the largest every rank supports) and synchronise the
    ghosts.  Returns the depth; `timings` (optional) receives the host time
    of each phase in ms."""
    t = [time.perf_counter()]
    blob = export_handles(b)
    t.append(time.perf_counter())
    blobs = gather_handles(blob, rank, world, all_gather_object)
    t.append(time.perf_counter())
    lo, hi = neighbours(rank, world)
    attach(b, blobs[lo] if lo is not None else None, blobs[hi] if hi is not None else None)
    d = temporal_depth(blobs) if depth is None else int(depth)
    if world > 1:
        set_depth(b, d)
    t.append(time.perf_counter())
    halo_sync(b, barrier)
    t.append(time.perf_counter())
    if timings is not None:
        for k, name in enumerate(("export", "gather", "attach", "halo_sync")):
            timings[name] = (t[k + 1] - t[k]) * 1e3
    return d if world > 1 else 1


class LocalSlabGroup:
    """Several slab contexts of one grid on one GPU, advanced in lockstep.

    depth: steps per exchange (1 or 2); None takes 2 when every context
    accepts it, else 1."""

    def __init__(self, backends: Sequence[GpuBackend3D], depth: Optional[int] = None):
        self.backends = list(backends)
        if not self.backends:
            raise ValueError("empty group")
        stream = self.backends[0].stream_handle()
        for b in self.backends[1:]:
            b.set_stream(stream)
        for i, b in enumerate(self.backends):
            lo = self.backends[i - 1]._ctx if i > 0 else None
            hi = self.backends[i + 1]._ctx if i + 1 < len(self.backends) else None
            b._chk(b._lib.ws3d_halo_attach_local(b._ctx, lo, hi), "halo_attach_local")
        self.depth = 1
        if len(self.backends) > 1:
            want = 2 if depth is None else int(depth)
            if want == 2 and not all(b._lib.ws3d_halo_set_depth(b._ctx, 2) == _ffi.WS3D_OK
                                     for b in self.backends):
                if depth is not None:
                    raise ValueError("temporal depth 2 is not possible for these slabs")
                want = 1
            for b in self.backends:
                set_depth(b, want)
            self.depth = want
        self.sync()

    def sync(self) -> None:
        for b in self.backends:
            b._chk(b._lib.ws3d_halo_sync(b._ctx, 0), "halo_sync(0)")
        for b in self.backends:
            b._chk(b._lib.ws3d_halo_sync(b._ctx, 1), "halo_sync(1)")

    def step_n(self, n: int) -> None:
        arr = (C.c_void_p * len(self.backends))(*[b._ctx.value for b in self.backends])
        b0 = self.backends[0]
        b0._chk(b0._lib.ws3d_step_group(arr, len(self.backends), int(n)), "step_group")

    def close(self) -> None:
        # The group shares the first context's stream: give every context its
        # own stream back before any of them (and that stream) is destroyed.
        for b in self.backends:
            if b._ctx:
                b.set_stream(None)
        for b in self.backends:
            b.close()
