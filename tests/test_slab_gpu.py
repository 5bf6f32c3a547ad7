"""z-slab decomposition on the GPU.

- Same-device slab groups (2-4 slabs, stream-ordered exchange) equal one
  context bit for bit, with sources and impulses on slab boundary planes.
- The bounded device wait gives up with WS3D_ETIMEOUT when a neighbour never
  raises its flag (a child process exports a slab that never steps), and the
  context stays usable.
- On a box with >= 2 GPUs: one process per GPU with the in-kernel NVLink
  exchange equals one GPU bit for bit.
"""
import multiprocessing as mpm
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from rustcompute_b200 import GpuBackend3D, TimeoutError_, _ffi, configs
from rustcompute_b200.slab import LocalSlabGroup, attach, export_handles, slab_bounds

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def make(wl, zb, ze, device=0, budget_ns=0, variant="auto"):
    whole = (zb, ze) == (0, wl.D)
    b = GpuBackend3D.create(wl.W, wl.H, wl.D, c_squared=wl.c_squared, damping=wl.damping,
                            device=device, variant=variant, sponge_width=wl.sponge_width,
                            sponge_max=wl.sponge_max, z_begin=0 if whole else zb,
                            z_end=0 if whole else ze, spin_budget_ns=budget_ns)
    p, pp = wl.initial_fields(zb, ze)
    b.upload_fields(p, pp)
    c2 = wl.c2_field(zb, ze)
    if c2 is not None:
        b.set_c2_field(c2)
    if len(wl.sources):
        b.set_sources(wl.sources, wl.wavelet)
    return b


@pytest.mark.parametrize("variant", ["auto", "zstream", "tma", "tma2"])
@pytest.mark.parametrize("nslab", [2, 3, 4])
@pytest.mark.parametrize("name,grid,steps", [("c3", (96, 72, 64), 50), ("c2", (48, 40, 37), 60),
                                             ("c3", (160, 40, 45), 31), ("c2", (264, 24, 70), 24)])
def test_local_slab_group_equals_single_context(nslab, name, grid, steps, variant):
    W, H, D = grid
    tma_ok = W > 128 and H >= 16
    two_ok = tma_ok and H >= _ffi.WS3D_TWO_STEP_ROWS + 4
    if variant in ("tma", "tma2") and not tma_ok:
        pytest.skip("TMA kernels need W > 128 and H >= 16")
    wl = configs.build(name, W, H, D, steps=steps)
    bounds = [slab_bounds(D, nslab, r) for r in range(nslab)]
    # put extra sources exactly on slab boundary planes (both sides)
    extra = [[W // 2, H // 2, bounds[1][0]], [W // 3, H // 3, bounds[0][1] - 1]]
    src = np.concatenate([wl.sources, np.array(extra, np.uint32)])
    wav = np.concatenate([wl.wavelet, np.tile(wl.wavelet[:1], (2, 1))])
    wl.sources, wl.wavelet = src, wav
    full = make(wl, 0, D)
    slabs = [make(wl, zb, ze, variant=variant) for zb, ze in bounds]
    grp = LocalSlabGroup(slabs)
    # two steps per exchange wherever the two-step kernel runs
    assert grp.depth == (2 if variant in ("auto", "tma2") and two_ok else 1)
    full.step_n(None, steps // 2)
    grp.step_n(steps // 2)
    for b in [full] + slabs:   # impulses on boundary planes
        b.inject_impulse(W // 4, H // 4, bounds[1][0], 0.5)
        b.inject_spherical_impulse(W // 2, H // 2, bounds[-1][0], 0.2, 2.5)
    grp.sync()                  # impulses changed boundary planes: re-sync ghosts
    full.step_n(None, steps - steps // 2)
    grp.step_n(steps - steps // 2)
    fp, fpp = full.download_field(with_prev=True)
    gp = np.concatenate([b.download_field() for b in slabs])
    gpp = np.concatenate([b.download_field(with_prev=True)[1] for b in slabs])
    assert np.array_equal(gp.view(np.uint32), fp.view(np.uint32))
    assert np.array_equal(gpp.view(np.uint32), fpp.view(np.uint32))
    grp.close()
    full.close()


def _idle_lower_neighbour(conn, grid, zb, ze):
    """Child process: owns the lower slab, exports it, never steps (its
    flags stay 0, so the parent's wait for the lower neighbour runs out)."""
    sys.path.insert(0, ROOT)
    from rustcompute_b200 import configs as cfg
    from rustcompute_b200.slab import export_handles as exp
    W, H, D = grid
    wl = cfg.build("c1", W, H, D, steps=4)
    b = make(wl, zb, ze)
    conn.send(exp(b))
    conn.recv()   # wait until the parent is done
    b.close()


@pytest.mark.parametrize("grid", [(64, 40, 48), (160, 40, 48)])  # z-stream / TMA kernel
def test_bounded_wait_times_out_and_context_stays_usable(grid):
    W, H, D = grid
    wl = configs.build("c1", W, H, D, steps=4)
    ctx = mpm.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_idle_lower_neighbour, args=(child, grid, 0, 24))
    proc.start()
    try:
        lower = parent.recv()
        b = make(wl, 24, 48, budget_ns=200_000_000)   # 0.2 s budget
        attach(b, lower, None)
        b._chk(b._lib.ws3d_halo_sync(b._ctx, 0), "sync0")
        b._chk(b._lib.ws3d_halo_sync(b._ctx, 1), "sync1")
        t0 = time.time()
        b.step_n(None, 1)
        with pytest.raises(TimeoutError_):
            b.sync()
        assert time.time() - t0 < 30
        # the waits that gave up are accounted: each ran for its whole budget
        ns, n = b.halo_wait_stats(reset=True)
        assert n >= 1 and ns >= n * 150_000_000, (ns, n)
        assert b.halo_wait_stats() == (0, 0)
        # the status was reported and cleared; the context still works
        b.sync()
        assert np.isfinite(b.energy())
        b.close()
    finally:
        parent.send("done")
        proc.join(timeout=60)
    assert proc.exitcode == 0


def _gpu_count():
    import torch
    return torch.cuda.device_count()


@pytest.mark.multigpu
@pytest.mark.parametrize("name,grid,steps,persistent", [("c3", "96x80x64", 60, False),
                                                        ("c2", "64x48x45", 50, False),
                                                        ("c5", "128x128x128", 200, True),
                                                        ("c3", "160x64x64", 40, True),
                                                        ("c3", "160x64x64", 41, False),
                                                        ("c2", "264x24x70", 30, "mixed")])
def test_multi_process_nvlink_slabs_equal_one_gpu(name, grid, steps, persistent):
    n = _gpu_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    n = min(n, 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(29400 + os.getpid() % 1000),
           os.path.join(ROOT, "tests", "mp_slab_check.py"), "--workload", name, "--grid", grid,
           "--steps", str(steps)] + (["--persistent"] if persistent is True else []) + \
        (["--mixed"] if persistent == "mixed" else [])
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, capture_output=True, text=True,
                       env=env)
    assert r.returncode == 0 and "SLAB-CHECK OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("nslab,grid", [(3, (264, 24, 40)), (4, (160, 40, 9)), (2, (300, 21, 30))])
def test_two_step_slabs_ghost_plane_sources_odd_counts_and_impulses(nslab, grid):
    """Temporal depth 2 on same-device slabs: sources on every plane next to
    a slab boundary (the ghost planes the kernel computes p_{t+1} on), odd
    step counts (single steps storing two planes), impulses on the two edge
    planes of each side between calls (mirrored two deep, no re-sync), c2
    field and sponge.  Bit-identical to one context."""
    W, H, D = grid
    wl = configs.build("c3", W, H, D, steps=8)
    bounds = [slab_bounds(D, nslab, r) for r in range(nslab)]
    pts = []
    for zb, _ in bounds[1:]:
        for dz in (-2, -1, 0, 1):
            pts.append([(W // 3 + 7 * dz) % W, (H // 2 + dz) % H, zb + dz])
    pts.append(pts[1])                     # a coinciding pair on a ghost plane
    rng = np.random.default_rng(D)
    wl.sources = np.array(pts, np.uint32)
    wl.wavelet = rng.standard_normal((len(pts), 11)).astype(np.float32)
    full = make(wl, 0, D)
    slabs = [make(wl, zb, ze) for zb, ze in bounds]
    grp = LocalSlabGroup(slabs)
    assert grp.depth == 2
    for n, dz in ((5, 0), (6, -1), (1, 1), (4, -2), (3, 0)):
        full.step_n(None, n)
        grp.step_n(n)
        for zb, _ in bounds[1:]:
            for b in [full] + slabs:
                b.inject_impulse(W // 2, H // 3, zb + dz, 0.4)
                b.inject_spherical_impulse(W // 4, H // 2, zb - 1, -0.3, 2.0)
    full.step_n(None, 7)
    grp.step_n(7)
    # same-device slabs are ordered by the stream: no device-side waits at all
    assert all(b.halo_wait_stats() == (0, 0) for b in slabs)
    fp, fpp = full.download_field(with_prev=True)
    gp = np.concatenate([b.download_field() for b in slabs])
    gpp = np.concatenate([b.download_field(with_prev=True)[1] for b in slabs])
    assert float(np.max(np.abs(fp))) > 1e-3
    assert np.array_equal(gp.view(np.uint32), fp.view(np.uint32)), int((gp != fp).sum())
    assert np.array_equal(gpp.view(np.uint32), fpp.view(np.uint32))
    grp.close()
    full.close()
