"""Multi-GPU host logic on CPU: z-slab bounds, the handle exchange over
torch.distributed (gloo, world sizes 2 and 3), the temporal-depth decision,
and slab-split emulations of the step with explicit ghost-plane exchange
(one step per exchange; the two-step kernel's data flow; k steps with
k-plane halos for k = 1 .. 4) that must equal the single-domain oracle bit
for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from rustcompute_b200 import configs
from rustcompute_b200.slab import gather_handles, neighbours, slab_bounds

f32 = np.float32


def test_slab_bounds_cover_the_grid():
    for D in (2, 7, 64, 512, 1023):
        for world in (1, 2, 3, 4, 8):
            if D < world:
                with pytest.raises(ValueError):
                    slab_bounds(D, world, 0)
                continue
            spans = [slab_bounds(D, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == D
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1


def test_neighbours():
    assert neighbours(0, 1) == (None, None)
    assert neighbours(0, 3) == (None, 1)
    assert neighbours(1, 3) == (0, 2)
    assert neighbours(2, 3) == (1, None)


def slab_step(Pext, PP, c2, damping, sponge, z0, Dg):
    """One step on a slab: Pext has nz+2 planes (ghosts at both ends), PP nz
    planes; returns the new owned planes.  Same op order as the reference
    (grid3d.rs:250-256), vectorised in float32 (no contraction)."""
    nz, H, W = PP.shape
    out = PP.copy()
    if W >= 3 and H >= 3:
        C = Pext[1:-1, 1:-1, 1:-1]
        lap = (Pext[1:-1, 1:-1, :-2] + Pext[1:-1, 1:-1, 2:])
        lap = lap + Pext[1:-1, :-2, 1:-1]
        lap = lap + Pext[1:-1, 2:, 1:-1]
        lap = lap + Pext[:-2, 1:-1, 1:-1]
        lap = lap + Pext[2:, 1:-1, 1:-1]
        lap = lap - f32(6.0) * C
        c2i = c2[:, 1:-1, 1:-1] if c2.ndim == 3 else c2
        pn = (f32(2.0) * C - PP[:, 1:-1, 1:-1]) + c2i * lap
        v = pn * f32(damping)
        if len(sponge):
            zg = np.arange(z0, z0 + nz)[:, None, None]
            y = np.arange(1, H - 1)[None, :, None]
            x = np.arange(1, W - 1)[None, None, :]
            d = np.minimum.reduce([np.broadcast_to(a, v.shape) for a in
                                   (x, W - 1 - x, y, H - 1 - y, zg, Dg - 1 - zg)])
            m = d < len(sponge)
            v = np.where(m, v * sponge[np.minimum(d, len(sponge) - 1)], v).astype(np.float32)
        zg = np.arange(z0, z0 + nz)
        planes = (zg >= 1) & (zg <= Dg - 2)
        out[planes, 1:-1, 1:-1] = v[planes]
    # reference faces: absorber with reflection 0.1
    zg = np.arange(z0, z0 + nz)
    face_plane = (zg == 0) | (zg == Dg - 1)
    out[face_plane] *= f32(0.1)
    rest = ~face_plane
    out[rest, 0, :] *= f32(0.1)
    out[rest, -1, :] *= f32(0.1)
    if H > 2:
        out[rest, 1:-1, 0] *= f32(0.1)
        out[rest, 1:-1, -1] *= f32(0.1)
    return out


def _rank_main(rank, world, port, wl_args, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    import oracle
    name, W, H, D, steps = wl_args
    wl = configs.build(name, W, H, D, steps=steps)
    zb, ze = slab_bounds(D, world, rank)
    nz = ze - zb
    # handle exchange: fake blobs stand in for the IPC handle structs
    blobs = gather_handles(f"rank{rank}:{zb}-{ze}".encode(), rank, world, dist.all_gather_object)
    assert blobs == [f"rank{r}:{slab_bounds(D, world, r)[0]}-{slab_bounds(D, world, r)[1]}".encode()
                     for r in range(world)]
    p, pp = wl.initial_fields(zb, ze)
    P = p.reshape(nz, H, W).copy()
    PP = pp.reshape(nz, H, W).copy()
    c2 = wl.c2_field(zb, ze)
    c2 = f32(wl.c_squared) if c2 is None else c2.reshape(nz, H, W)
    sponge = oracle.sponge_table(wl.sponge_width, wl.sponge_max) if wl.sponge_width \
        else np.zeros(0, np.float32)
    lo, hi = neighbours(rank, world)
    for s in range(steps):
        for k, (x, y, z) in enumerate(wl.sources):
            if zb <= z < ze:
                a = wl.wavelet[k, s] if s < wl.wavelet.shape[1] else f32(0)
                P[z - zb, y, x] = P[z - zb, y, x] + a
                PP[z - zb, y, x] = PP[z - zb, y, x] + a * f32(0.5)
        Pext = np.zeros((nz + 2, H, W), np.float32)
        Pext[1:-1] = P
        # exchange boundary planes with the neighbours (gloo point-to-point)
        reqs = []
        if lo is not None:
            reqs.append(dist.isend(torch.from_numpy(P[0].copy()), lo))
        if hi is not None:
            reqs.append(dist.isend(torch.from_numpy(P[-1].copy()), hi))
        if lo is not None:
            t = torch.empty(H, W)
            dist.recv(t, lo)
            Pext[0] = t.numpy()
        if hi is not None:
            t = torch.empty(H, W)
            dist.recv(t, hi)
            Pext[-1] = t.numpy()
        for r in reqs:
            r.wait()
        new = slab_step(Pext, PP, c2, wl.damping, sponge, zb, D)
        P, PP = new, P
    out = [None] * world
    dist.all_gather_object(out, (zb, P.copy(), PP.copy()))
    if rank == 0:
        full_p = np.concatenate([o[1] for o in sorted(out, key=lambda t: t[0])]).reshape(-1)
        full_pp = np.concatenate([o[2] for o in sorted(out, key=lambda t: t[0])]).reshape(-1)
        ref = oracle.from_workload(wl)
        ref.run(steps, 1)
        result_q.put((bool(np.array_equal(full_p, ref.pressure)),
                      bool(np.array_equal(full_pp, ref.pressure_prev))))
    dist.barrier()
    dist.destroy_process_group()


def _exchange(t_lo, t_hi, lo, hi, shape):
    """Send t_lo to the lower neighbour and t_hi to the upper one; return what
    they sent us (lower's, upper's).  gloo point-to-point."""
    import torch
    reqs = []
    if lo is not None:
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(t_lo)), lo))
    if hi is not None:
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(t_hi)), hi))
    got_lo = got_hi = None
    if lo is not None:
        t = torch.empty(shape)
        dist.recv(t, lo)
        got_lo = t.numpy()
    if hi is not None:
        t = torch.empty(shape)
        dist.recv(t, hi)
        got_hi = t.numpy()
    for r in reqs:
        r.wait()
    return got_lo, got_hi


def _rank_main_depth2(rank, world, port, wl_args, result_q):
    """Temporal depth 2 on z-slabs, the data flow of k_step_tma2 on slabs:
    per pair of steps the ranks exchange two edge planes of p_t, and each
    rank gets its neighbours' own p_{t-1} and c2 edge planes; it computes
    p_{t+1} on its planes plus one ghost plane per side (sources of step t+1
    included), then p_{t+2} on its own planes.  An odd last step is a single
    step.  Must equal the single-domain oracle bit for bit."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    name, W, H, D, steps = wl_args
    wl = configs.build(name, W, H, D, steps=steps)
    zb, ze = slab_bounds(D, world, rank)
    nz = ze - zb
    lo, hi = neighbours(rank, world)
    p, pp = wl.initial_fields(zb, ze)
    P = p.reshape(nz, H, W).copy()
    PP = pp.reshape(nz, H, W).copy()
    c2f = wl.c2_field(zb, ze)
    C2 = np.full((nz, H, W), f32(wl.c_squared)) if c2f is None else c2f.reshape(nz, H, W)
    sponge = oracle.sponge_table(wl.sponge_width, wl.sponge_max) if wl.sponge_width \
        else np.zeros(0, np.float32)
    # the neighbours' c2 edge planes never change: fetch them once
    c2_lo, c2_hi = _exchange(C2[0], C2[-1], lo, hi, (H, W))
    xlo = -1 if lo is not None else 0           # X planes [xlo, xhi) in local z
    xhi = nz + 1 if hi is not None else nz

    def amp(k, s):
        return wl.wavelet[k, s] if s < wl.wavelet.shape[1] else f32(0)

    s = 0
    while s < steps:
        for k, (x, y, z) in enumerate(wl.sources.tolist()):   # sources of step s (host, own planes)
            if zb <= z < ze:
                P[z - zb, y, x] = P[z - zb, y, x] + amp(k, s)
                PP[z - zb, y, x] = PP[z - zb, y, x] + amp(k, s) * f32(0.5)
        # A: own planes plus two ghost planes per side (zeros beyond the grid)
        g_lo, g_hi = _exchange(P[:2], P[-2:], lo, hi, (2, H, W))
        A = np.zeros((nz + 4, H, W), np.float32)
        A[2:-2] = P
        if g_lo is not None:
            A[:2] = g_lo
        if g_hi is not None:
            A[-2:] = g_hi
        if steps - s == 1:   # single step
            new = slab_step(A[1:-1], PP, C2, wl.damping, sponge, zb, D)
            P, PP = new, P
            s += 1
            continue
        # B and c2 on planes [xlo, xhi): the neighbours' own edge planes
        b_lo, b_hi = _exchange(PP[0], PP[-1], lo, hi, (H, W))

        def ext(own, below, above):   # planes [xlo, xhi)
            return np.concatenate(([below[None]] if xlo < 0 else []) + [own] +
                                  ([above[None]] if xhi > nz else []))
        B = ext(PP, b_lo, b_hi)
        Cx = ext(C2, c2_lo, c2_hi)
        X = slab_step(A[xlo + 1:xhi + 3], B, Cx, wl.damping, sponge, zb + xlo, D)
        Pm = P.copy()                                  # p_prev of the second step
        for k, (x, y, z) in enumerate(wl.sources.tolist()):     # sources of step s+1
            if zb + xlo <= z < zb + xhi:
                X[z - zb - xlo, y, x] = X[z - zb - xlo, y, x] + amp(k, s + 1)
            if zb <= z < ze:
                Pm[z - zb, y, x] = Pm[z - zb, y, x] + amp(k, s + 1) * f32(0.5)
        Xe = np.zeros((nz + 2, H, W), np.float32)      # X on planes -1 .. nz
        Xe[1 + xlo:1 + xhi] = X
        Y = slab_step(Xe, Pm, C2, wl.damping, sponge, zb, D)
        P, PP = Y, X[-xlo:-xlo + nz]
        s += 2
    out = [None] * world
    dist.all_gather_object(out, (zb, P.copy(), PP.copy()))
    if rank == 0:
        full_p = np.concatenate([o[1] for o in sorted(out, key=lambda t: t[0])]).reshape(-1)
        full_pp = np.concatenate([o[2] for o in sorted(out, key=lambda t: t[0])]).reshape(-1)
        ref = oracle.from_workload(wl)
        ref.run(steps, 1)
        result_q.put((bool(np.array_equal(full_p, ref.pressure)),
                      bool(np.array_equal(full_pp, ref.pressure_prev))))
    dist.barrier()
    dist.destroy_process_group()


def _rank_main_depthk(rank, world, port, wl_args, k, result_q):
    """Temporal depth k on z-slabs with k-cell halos (k = 1 .. 4).  Per
    round of k steps a rank receives k edge planes of p_t and k-1 of p_{t-1}
    from each neighbour (the c2 edge planes once), computes level j =
    p_{t+j} on its planes plus k-j ghost planes per side that has a
    neighbour (sources of step t+j: level j += a, the next level's p_prev =
    level j-1 + a/2), and keeps levels k and k-1 of its own planes; a last
    round of depth steps % k finishes.  The GPU kernel builds k = 2; this
    pins the scheme for every k against the single-domain oracle."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    name, W, H, D, steps = wl_args
    wl = configs.build(name, W, H, D, steps=steps)
    zb, ze = slab_bounds(D, world, rank)
    nz = ze - zb
    lo, hi = neighbours(rank, world)
    p, pp = wl.initial_fields(zb, ze)
    P = p.reshape(nz, H, W).copy()
    PP = pp.reshape(nz, H, W).copy()
    c2f = wl.c2_field(zb, ze)
    C2 = np.full((nz, H, W), f32(wl.c_squared)) if c2f is None else c2f.reshape(nz, H, W)
    sponge = oracle.sponge_table(wl.sponge_width, wl.sponge_max) if wl.sponge_width \
        else np.zeros(0, np.float32)
    src = wl.sources.tolist()

    def amp(j, step):
        return wl.wavelet[j, step] if step < wl.wavelet.shape[1] else f32(0)

    def span(e):   # global planes of a level with e ghost planes per neighbour side
        return (zb - e if lo is not None else zb), (ze + e if hi is not None else ze)

    def with_ghosts(own, below, above, e):
        """(array, global start) of own planes plus e planes from each neighbour."""
        parts = ([below] if lo is not None and e else []) + [own] + \
            ([above] if hi is not None and e else [])
        return np.concatenate(parts), span(e)[0]

    def take(arr, start, z0, z1):
        """planes [z0, z1) of arr (first plane = global start), zeros outside it."""
        out = np.zeros((z1 - z0, H, W), np.float32)
        a, b = max(z0, start), min(z1, start + arr.shape[0])
        if b > a:
            out[a - z0:b - z0] = arr[a - start:b - start]
        return out

    def add_sources(arr, start, step, scale):
        for j, (x, y, z) in enumerate(src):
            if start <= z < start + arr.shape[0]:
                v = amp(j, step) if scale == 1 else amp(j, step) * f32(0.5)
                arr[z - start, y, x] = arr[z - start, y, x] + v

    g = max(k - 1, 0)
    c2_lo, c2_hi = _exchange(C2[:g], C2[nz - g:], lo, hi, (g, H, W))
    C2x, c2_start = with_ghosts(C2, c2_lo, c2_hi, g)
    s = 0
    while s < steps:
        d = min(k, steps - s)
        add_sources(P, zb, s, 1)                       # sources of step s (host, own planes)
        add_sources(PP, zb, s, 0.5)
        a_lo, a_hi = _exchange(P[:d], P[nz - d:], lo, hi, (d, H, W))
        b_lo, b_hi = _exchange(PP[:d - 1], PP[nz - d + 1:], lo, hi, (d - 1, H, W))
        lev = [with_ghosts(P, a_lo, a_hi, d)]           # (array, start) per level
        prev = with_ghosts(PP, b_lo, b_hi, d - 1)       # p_prev of level 1
        for j in range(1, d + 1):
            z0, z1 = span(d - j)
            src_arr, src_start = lev[j - 1]
            Pe = take(src_arr, src_start, z0 - 1, z1 + 1)
            pv = take(prev[0], prev[1], z0, z1)
            c2j = take(C2x, c2_start, z0, z1)
            out = slab_step(Pe, pv, c2j, wl.damping, sponge, z0, D)
            if j < d:
                add_sources(out, z0, s + j, 1)          # p_{s+j} += a
                nz0, nz1 = span(d - j - 1)
                nxt = take(src_arr, src_start, nz0, nz1)  # level j-1 as the next p_prev
                add_sources(nxt, nz0, s + j, 0.5)
                prev = (nxt, nz0)
            lev.append((out, z0))
        P = take(lev[d][0], lev[d][1], zb, ze)
        PP = take(lev[d - 1][0], lev[d - 1][1], zb, ze)   # holds its step s+d-1 sources
        s += d
    out = [None] * world
    dist.all_gather_object(out, (zb, P.copy(), PP.copy()))
    if rank == 0:
        full_p = np.concatenate([o[1] for o in sorted(out, key=lambda t: t[0])]).reshape(-1)
        full_pp = np.concatenate([o[2] for o in sorted(out, key=lambda t: t[0])]).reshape(-1)
        ref = oracle.from_workload(wl)
        ref.run(steps, 1)
        assert float(np.max(np.abs(ref.pressure))) > 1e-4   # a field worth comparing
        result_q.put((bool(np.array_equal(full_p, ref.pressure)),
                      bool(np.array_equal(full_pp, ref.pressure_prev))))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,wl_args", [
    (2, ("c3", 40, 36, 30, 25)),     # heterogeneous + sponge + centred source
    (3, ("c2", 34, 30, 33, 40)),     # sources + sponge
    (2, ("c1", 24, 20, 2, 5)),       # one plane per slab: both planes are faces
])
def test_gloo_slab_emulation_matches_oracle(world, wl_args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, wl_args, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    assert q.get(timeout=5) == (True, True)


@pytest.mark.parametrize("world,wl_args", [
    (2, ("c3", 40, 36, 30, 25)),     # heterogeneous + sponge + centred source, odd steps
    (3, ("c2", 34, 30, 33, 40)),     # sources (also on ghost planes) + sponge
    (3, ("c1", 24, 20, 7, 6)),       # 2-3 planes per slab: pushes reach both neighbours
])
def test_gloo_two_step_slab_emulation_matches_oracle(world, wl_args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_depth2, args=(r, world, port, wl_args, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    assert q.get(timeout=5) == (True, True)


def _blob(zb, ze, caps, c2=0.25):
    from rustcompute_b200 import _ffi
    h = _ffi.ws3d_halo_handles()
    h.z_begin, h.z_end, h.caps, h.c_squared, h.ghost_planes = zb, ze, caps, c2, 2
    return bytes(h)


def test_temporal_depth_is_decided_from_every_rank():
    from rustcompute_b200 import _ffi
    from rustcompute_b200.slab import temporal_depth
    T, F = _ffi.HALO_CAP_TWO_STEP, _ffi.HALO_CAP_C2_FIELD
    assert temporal_depth([_blob(0, 8, T), _blob(8, 16, T)]) == 2
    assert temporal_depth([_blob(0, 8, T | F), _blob(8, 16, T | F)]) == 2
    assert temporal_depth([_blob(0, 8, T), _blob(8, 16, 0)]) == 1          # one rank cannot
    assert temporal_depth([_blob(0, 8, T), _blob(8, 9, T), _blob(9, 16, T)]) == 1  # 1-plane slab
    assert temporal_depth([_blob(0, 8, T | F), _blob(8, 16, T)]) == 1      # c2 field on one side
    assert temporal_depth([_blob(0, 8, T, 0.25), _blob(8, 16, T, 0.2)]) == 1  # other uniform c2
    assert temporal_depth([_blob(0, 16, T)]) == 1


@pytest.mark.parametrize("k", [1, 2, 3, 4])
@pytest.mark.parametrize("world,wl_args", [
    (3, ("c2", 34, 30, 33, 23)),     # sources (on ghost planes too) + sponge, 23 steps: ragged last round
    (2, ("c3", 40, 36, 30, 18)),     # heterogeneous + sponge + centred source
])
def test_gloo_depth_k_slab_emulation_matches_oracle(world, wl_args, k):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main_depthk, args=(r, world, port, wl_args, k, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    assert q.get(timeout=5) == (True, True)
