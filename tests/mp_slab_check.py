"""Multi-GPU z-slab check, one process per GPU (run by tests/test_slab_gpu.py
through torchrun).  Every rank steps its slab with the in-kernel NVLink halo
exchange; rank 0 gathers the slabs and compares them, bit for bit, with a
single-GPU run of the same workload.  Prints "SLAB-CHECK OK" on success.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 tests/mp_slab_check.py \
        --workload c3 --grid 96x80x64 --steps 60
"""
import argparse
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="c3")
    ap.add_argument("--grid", default="96x80x64")
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--persistent", action="store_true",
                    help="advance the slabs with ws3d_step_persistent")
    ap.add_argument("--mixed", action="store_true",
                    help="persistent steps first (one edge plane per side), then ws3d_step")
    args = ap.parse_args()
    import torch
    import torch.distributed as dist

    from rustcompute_b200 import GpuBackend3D, configs
    from rustcompute_b200.slab import connect, slab_bounds

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    W, H, D = (int(v) for v in args.grid.split("x"))
    wl = configs.build(args.workload, W, H, D, steps=args.steps)
    zb, ze = slab_bounds(D, world, rank)

    def make(z_begin, z_end, device):
        whole = (z_begin, z_end) == (0, D)
        b = GpuBackend3D.create(W, H, D, c_squared=wl.c_squared, damping=wl.damping,
                                device=device, sponge_width=wl.sponge_width,
                                sponge_max=wl.sponge_max, z_begin=0 if whole else z_begin,
                                z_end=0 if whole else z_end)
        p, pp = wl.initial_fields(z_begin, z_end)
        b.upload_fields(p, pp)
        c2 = wl.c2_field(z_begin, z_end)
        if c2 is not None:
            b.set_c2_field(c2)
        if len(wl.sources):
            b.set_sources(wl.sources, wl.wavelet)
        return b

    b = make(zb, ze, local)
    depth = connect(b, rank, world, dist.all_gather_object, dist.barrier)
    # Impulses on both sides of every slab boundary exercise the ghost updates.
    for r in range(1, world):
        zc = slab_bounds(D, world, r)[0]
        b.inject_impulse(W // 3, H // 2, zc, 0.25)
        b.inject_impulse(W // 2, H // 3, zc - 1, -0.5)
    adv = b.step_persistent if args.persistent else (lambda n: b.step_n(None, n))
    (b.step_persistent if args.mixed else adv)(7)
    b.inject_spherical_impulse(W // 2, H // 2, slab_bounds(D, world, world // 2)[0], 0.3, 3.0)
    adv(args.steps - 7)
    b.sync()
    p, pp = b.download_field(with_prev=True)
    parts = [None] * world
    dist.all_gather_object(parts, (zb, p, pp))
    ok = True
    if rank == 0:
        full = make(0, D, local)
        for r in range(1, world):
            zc = slab_bounds(D, world, r)[0]
            full.inject_impulse(W // 3, H // 2, zc, 0.25)
            full.inject_impulse(W // 2, H // 3, zc - 1, -0.5)
        full.step_n(None, 7)
        full.inject_spherical_impulse(W // 2, H // 2, slab_bounds(D, world, world // 2)[0], 0.3, 3.0)
        full.step_n(None, args.steps - 7)
        fp, fpp = full.download_field(with_prev=True)
        parts.sort(key=lambda t: t[0])
        gp = np.concatenate([t[1] for t in parts])
        gpp = np.concatenate([t[2] for t in parts])
        ok = np.array_equal(gp.view(np.uint32), fp.view(np.uint32)) and \
            np.array_equal(gpp.view(np.uint32), fpp.view(np.uint32))
        nbad = int(np.count_nonzero(gp != fp))
        print(f"SLAB-CHECK {'OK' if ok else 'FAIL'} world={world} grid={args.grid} "
              f"steps={args.steps} depth={depth} differing cells={nbad}", flush=True)
        full.close()
    b.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
