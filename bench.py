#!/usr/bin/env python
"""Benchmark of the B200 WaveSim3D FDTD step (BASELINE config 3 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c3] [--variant zstream]

One "step" is one FDTD time step of the whole grid.  Rank 0 prints one JSON
line.  For N > 1 the script runs under torchrun, one rank per GPU, each rank
owning a z-slab of the grid: by default one full-size slab of the recipe per
GPU (weak scaling, grid W x H x D*N); --scaling strong splits the
single-GPU grid instead.

value     global cells x K / device time of the K timed steps (CUDA events on
          the launch stream, max over ranks), fields resident in HBM.
e2e       the same metric for a whole job through the public API with pinned
          host buffers: upload p, p_prev, c2 and the source wavelets, K steps,
          download p -- all inside the timed region.
roofline  algorithmic bytes per step-kernel launch / its average duration,
          against MEASURED_PEAKS.json: 12 B/cell (16 B with a c2 field) for a
          one-step launch; read p, p_prev (+ c2) and write two fields, 16 B/cell
          (20 B with c2), for a two-step launch (variant tma2).
cpu_baseline  the C restatement of the reference CPU step (oracle/, "port")
          timed on this host's cores over a bounded sample (rank 0, N = 1).
--impl reference  the reference's CPU implementation of the path (the same
          C restatement: the Rust crate cannot be built here) on this host's
          cores, same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from rustcompute_b200.slab import slab_bounds  # noqa: E402

METRIC = "Mcells/s and % HBM roofline at 1/2/4/8 B200 (3D FDTD step) vs host CPU"
UNIT = "Mcells/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c3")
    ap.add_argument("--variant", default="auto",
                    help="auto (TMA pipeline on one GPU, z-stream for z-slabs), tma, zstream, "
                         "naive, refshape")
    ap.add_argument("--mode", default="step", choices=["step", "persistent", "resident"],
                    help="step: one launch per step (library-timed); persistent: all K steps "
                         "in one cooperative launch (config 5); resident: one resident kernel "
                         "driven by a RUN_STEPS command (host wall clock from the command to "
                         "the kernel reporting the last step; one GPU)")
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="N > 1: weak (default) keeps one D-plane slab of the recipe per GPU "
                         "(grid W x H x D*N, as BASELINE config 4's weak scaling); strong "
                         "splits the single-GPU grid into N slabs")
    ap.add_argument("--grid", default=None,
                    help="WxHxD: the workload's recipe at another size (profiling cases)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--comparators", action="store_true",
                    help="also time the naive and reference-shaped kernels")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def ncu_traffic(wl, kernel: str):
    """DRAM bytes per launch of the step kernel from a committed ncu summary
    (profiles/traffic.json, keyed by workload, grid and kernel), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    e = d.get(f"{wl.name}/{wl.W}x{wl.H}x{wl.D}/{kernel}")
    return None if e is None else e.get("dram_bytes_per_launch")


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML (read-only)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device: int, period_s: float = 0.02):
        self.samples, self.reasons = [], 0
        self.period = period_s
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def cpu_sample_run(wl, target_s: float = 12.0, nthreads: int = 0):
    """Time the oracle (CPU port of the reference step, OpenMP over z-planes
    like step_parallel) on a bounded sample of the workload: full-grid steps
    filling ~target_s when one step takes < target_s/3, else a z-slab of the
    same recipe."""
    import oracle
    nthreads = nthreads or host_threads()
    g = oracle.from_workload(wl)
    # Step counts stay even: an odd count makes the oracle copy the fields
    # back into the caller's arrays, which would be timed with the steps.
    g.run(2, nthreads)                     # warm-up (first touch, thread pool)
    # calibration: steady-state seconds per step over at least ~1 s of steps
    n, t0 = 0, time.perf_counter()
    while True:
        g.run(2, nthreads)
        n += 2
        t1 = (time.perf_counter() - t0) / n
        if n * t1 >= 1.0 or t1 * 3 > target_s:
            break
    if t1 * 3 <= target_s:
        steps = max(2, int(target_s / max(t1, 1e-6)) // 2 * 2)
        sample = f"{steps} full {wl.W}x{wl.H}x{wl.D} steps after {2 + n} untimed steps"
        cells = wl.cells
    else:
        planes = max(8, min(wl.D, int(wl.D * target_s / 3 / t1)))
        sub = wl.scaled(wl.W, wl.H, planes, steps=4)
        g = oracle.from_workload(sub)
        g.run(1, nthreads)
        steps, cells = 2, sub.cells
        sample = (f"2 steps of a {wl.W}x{wl.H}x{planes} slab of the {wl.name} recipe "
                  "(same per-cell work) after 1 untimed step")
    t0 = time.perf_counter()
    g.run(steps, nthreads)
    dt = time.perf_counter() - t0
    return cells * steps / dt / 1e6, nthreads, sample, dt


def run_reference(args, wl):
    """--impl reference: the reference's CPU path (C restatement) on host cores."""
    import oracle
    rank, world, _ = dist_env()
    if rank != 0:
        return
    nthreads = host_threads()
    # One timed step = one full-grid step when affordable, else a z-slab sample.
    probe = wl.scaled(wl.W, wl.H, min(wl.D, 34), steps=4)
    g = oracle.from_workload(probe)
    g.run(2, nthreads)                     # warm-up; even counts: no copy-back
    t0 = time.perf_counter()
    g.run(2, nthreads)
    rate = 2 * probe.cells / max(time.perf_counter() - t0, 1e-9)
    budget = 150.0 / max(args.steps + args.warmup, 1)
    if wl.cells / rate <= budget:
        sample, desc = wl, f"full {wl.W}x{wl.H}x{wl.D} grid per step"
    else:
        planes = max(8, min(wl.D, int(budget * rate / (wl.W * wl.H))))
        sample = wl.scaled(wl.W, wl.H, planes, steps=args.steps + args.warmup + 1)
        desc = f"{wl.W}x{wl.H}x{planes} z-slab of the {wl.name} recipe per step (bounded sample)"
    g = oracle.from_workload(sample)
    g.run(args.warmup, nthreads)
    t0 = time.perf_counter()
    g.run(args.steps, nthreads)
    dt = time.perf_counter() - t0
    val = sample.cells * args.steps / dt / 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SplitMix64 medium and sources)",
        "config": {"workload": wl.name, "grid": [wl.W, wl.H, wl.D],
                   "heterogeneous": wl.heterogeneous, "sponge": wl.sponge_width,
                   "sources": int(len(wl.sources))},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference Rust crate cannot be built in this image (no cargo, wgpu "
                "dependency); this arm times its CPU step restated in C (oracle/)",
    }
    emit(line)


def make_backend(wl, variant, device, zb, ze):
    from rustcompute_b200 import GpuBackend3D
    whole = (zb, ze) == (0, wl.D)
    return GpuBackend3D.create(wl.W, wl.H, wl.D, c_squared=wl.c_squared, damping=wl.damping,
                               device=device, variant=variant, sponge_width=wl.sponge_width,
                               sponge_max=wl.sponge_max, z_begin=0 if whole else zb,
                               z_end=0 if whole else ze)


def upload_inputs(b, wl, p, pp, c2):
    """The job's host inputs: both fields, the medium and the source wavelets."""
    b.upload_fields(p, pp)
    if c2 is not None:
        b.set_c2_field(c2)
    if len(wl.sources):
        b.set_sources(wl.sources, wl.wavelet)


def pinned(a):
    import torch
    if a is None:
        return None
    t = torch.empty(a.size, dtype=torch.float32, pin_memory=True)
    t.numpy()[:] = a
    return t.numpy()


def kernel_name(variant, wl, world, mode="step", depth=1):
    """The step kernel the library runs; on z-slabs two-step launches need
    temporal depth 2 (`depth`, as negotiated by slab.connect)."""
    if mode == "persistent":
        return "k_persistent"
    if mode == "resident":
        return "k_resident"
    if variant in ("auto", "tma2"):   # mirrors the library's choice for the default faces
        tma_ok = wl.W > 128 and wl.H >= 16
        two_step = (world == 1 or depth == 2) and tma_ok and len(wl.sources) <= 32 and \
            wl.sponge_width <= 64
        variant = "tma2" if two_step else ("tma" if tma_ok else "zstream")
    return {"tma": "k_step_tma", "tma2": "k_step_tma2", "async": "k_step_async",
            "zstream": "k_step_zstream",
            "naive": "k_step_naive", "refshape": "k_ref_stencil+k_ref_boundary"}[variant]


def run_ours(args, wl):
    import datetime

    import torch
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    zb, ze = slab_bounds(wl.D, world, rank)
    local_cells = (ze - zb) * wl.W * wl.H

    def barrier():
        if pg is not None:
            pg.barrier()

    def max_over_ranks(v: float) -> float:
        if pg is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.Stream(device=dev)   # a real stream (handle != 0) shared with the library
    p0, pp0 = wl.initial_fields(zb, ze)
    c20 = wl.c2_field(zb, ze)

    def open_backend():
        b = make_backend(wl, args.variant, local, zb, ze)
        b.set_stream(stream.cuda_stream)
        return b

    b = open_backend()
    upload_inputs(b, wl, p0, pp0, c20)
    depth = 1   # steps per halo exchange on z-slabs
    if world > 1:
        from rustcompute_b200.slab import connect
        depth = connect(b, rank, world, pg.all_gather_object, barrier)

    # Warm-up (>= 3 steps), then the timed region: K steps between two events
    # on the launch stream; the library also times every step-kernel launch.
    b.step_n(None, max(args.warmup, 3))
    b.sync()
    if args.mode == "resident":
        if world != 1:
            raise SystemExit("--mode resident runs on one GPU")
        from rustcompute_b200 import _ffi
        import ctypes as C
        cfg = _ffi.ws3d_resident_config(progress_interval=1 << 62, idle_budget_ns=2_000_000_000)
        b._chk(b._lib.ws3d_resident_start(b._ctx, C.byref(cfg)), "resident_start")
        st0 = b.stats()["step"]
        b._chk(b._lib.ws3d_resident_run_steps(b._ctx, max(args.warmup, 3)), "run_steps")
        b._chk(b._lib.ws3d_resident_wait_step(b._ctx, st0 + max(args.warmup, 3), 0), "wait")
    launches0 = b.stats()["kernel_launches"]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        e0.record(stream)
        if args.mode == "resident":
            rs = _ffi.ws3d_resident_stats()
            b._chk(b._lib.ws3d_resident_stats_get(b._ctx, C.byref(rs)), "resident_stats")
            t0 = time.perf_counter()
            b._chk(b._lib.ws3d_resident_run_steps(b._ctx, args.steps), "run_steps")
            b._chk(b._lib.ws3d_resident_wait_step(b._ctx, rs.current_step + args.steps, 0),
                   "wait")
            host_ms = (time.perf_counter() - t0) * 1e3
            b._chk(b._lib.ws3d_resident_shutdown(b._ctx, 0), "resident_shutdown")
            e1.record(stream)
            kernel_ms = None
        elif args.mode == "persistent":
            b.step_persistent(args.steps)
            e1.record(stream)
            b.sync()
            kernel_ms = None
        else:
            kernel_ms = b.step_timed(args.steps)   # synchronises the stream at the end
            e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    launches = b.stats()["kernel_launches"] - launches0
    total_ms = max_over_ranks(host_ms if args.mode == "resident" else e0.elapsed_time(e1))
    value = wl.cells * args.steps / (total_ms * 1e-3) / 1e6

    if kernel_ms is None:   # persistent / resident: the one launch is the whole timed region
        kernel_ms = total_ms
    bpc = wl.bytes_per_cell_step
    kname = kernel_name(args.variant, wl, world, args.mode, depth)
    if kname == "k_step_tma2" and args.mode == "step":
        # K // 2 two-step launches (+ one single step for odd K)
        n_launch = args.steps // 2 + args.steps % 2
        total_bytes = ((args.steps // 2) * (bpc + 4) + (args.steps % 2) * bpc) * local_cells
        alg_bytes = (bpc + 4) * local_cells
    else:
        n_launch = args.steps
        total_bytes = bpc * local_cells * args.steps
        alg_bytes = bpc * local_cells
    avg_kernel_ms = kernel_ms / n_launch
    peaks = measured_peaks()
    achieved = total_bytes / (kernel_ms * 1e-3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"],
                "traffic": ncu_traffic(wl, kernel_name(args.variant, wl, world, depth=depth)),
                "algorithmic_bytes_per_launch": alg_bytes,
                "steps_per_launch": 2 if kname == "k_step_tma2" and args.mode == "step" else 1,
                # algorithmic bytes per cell of one launch: one step moves bpc (read p,
                # p_prev (+ c2), write one field); a two-step launch bpc + 4 (one more write)
                "bytes_per_cell_per_launch": alg_bytes // max(local_cells, 1),
                "bytes_per_cell_step": bpc,
                "kernel_avg_ms": avg_kernel_ms,
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"
                               if peaks["source"] == "measured" else "fallback",
                "kernel": kernel_name(args.variant, wl, world, args.mode, depth),
                "rank": rank}

    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SplitMix64 medium and sources)",
        "config": {"workload": wl.name, "grid": [wl.W, wl.H, wl.D], "variant": args.variant,
                   "heterogeneous": wl.heterogeneous, "sponge": wl.sponge_width,
                   "sources": int(len(wl.sources)), "decomposition": f"z-slabs x{world}",
                   "halo_depth": depth,
                   "l2": "inputs larger than L2 (each field %d MiB > 126 MB)"
                         % (wl.cells * 4 // 2 ** 20)},
        "us_per_step": total_ms * 1e3 / args.steps,
        "mode": args.mode,
        "timing": ("host wall clock from the RUN_STEPS command to the kernel reporting the last "
                   "step (the resident kernel owns the stream)") if args.mode == "resident"
                  else "CUDA events on the launch stream",
        "roofline": roofline,
        "clocks": clk.summary(),
        "gpu_launches": int(launches),
    }
    b.close()

    # e2e: one whole job through the public API with pinned host buffers.
    if not args.no_e2e:
        pins = [pinned(a) for a in (p0, pp0, c20)]
        outp = pinned(np.zeros(local_cells, np.float32))
        h2d = sum(a.nbytes for a in pins if a is not None)
        h2d += (wl.wavelet.nbytes + wl.sources.nbytes) if len(wl.sources) else 0
        d2h = outp.nbytes
        b2 = open_backend()
        barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        upload_inputs(b2, wl, *pins)            # synchronous
        t1 = time.perf_counter()
        conn = {}
        if world > 1:
            from rustcompute_b200.slab import connect
            connect(b2, rank, world, pg.all_gather_object, barrier, timings=conn)
        t2 = time.perf_counter()
        b2.step_n(None, args.steps)
        b2.sync()                               # the download would wait for the steps anyway
        t3 = time.perf_counter()
        b2.download_into(outp)
        t4 = time.perf_counter()
        e2e_ms = max_over_ranks((t4 - t0) * 1e3)
        phases = {k: max_over_ranks(v * 1e3) for k, v in
                  (("upload", t1 - t0), ("connect", t2 - t1), ("steps", t3 - t2),
                   ("download", t4 - t3))}
        for k in ("export", "gather", "attach", "halo_sync"):   # same calls on every rank
            if world > 1:
                phases["connect_" + k] = max_over_ranks(conn[k])
        result["e2e"] = {"value": wl.cells * args.steps / (e2e_ms * 1e-3) / 1e6, "unit": UNIT,
                         "h2d_bytes_per_step": h2d * world // args.steps,
                         "d2h_bytes_per_step": d2h * world // args.steps,
                         "job": f"upload p, p_prev{', c2' if wl.heterogeneous else ''}"
                                f"{', source wavelets' if len(wl.sources) else ''} from pinned "
                                f"host memory; {args.steps} steps; download p"
                                f"{'; slab handle exchange' if world > 1 else ''}",
                         "job_ms": e2e_ms, "phases_ms": phases,
                         "clock": "host wall clock, max over ranks"}
        b2.close()

    if args.comparators and world == 1:
        comps = {}
        for v in ("async", "zstream", "naive", "refshape"):
            bc = make_backend(wl, v, local, zb, ze)
            bc.set_stream(stream.cuda_stream)
            upload_inputs(bc, wl, p0, pp0, c20)
            bc.step_n(None, 3)
            n = max(10, min(args.steps, 50))
            ms = bc.step_timed(n)
            comps[v] = {"value": wl.cells * n / (ms * 1e-3) / 1e6, "unit": UNIT, "steps": n,
                        "note": "step-kernel time only"}
            bc.close()
        result["comparators"] = comps

    if rank == 0 and world == 1 and not args.no_cpu:
        val, cores, desc, secs = cpu_sample_run(wl)
        result["cpu_baseline"] = {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
                                  "sample": desc, "seconds": secs}
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0:
        emit(result)


def host_threads() -> int:
    """Host cores this process may use (torchrun sets OMP_NUM_THREADS=1 for
    its ranks; the CPU legs use every core they are allowed to run on)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


_JSON_OUT = None


def emit(line: dict) -> None:
    """Write the result line to the real stdout (libraries such as NCCL may
    print banners to fd 1; main() points fd 1 at stderr for them)."""
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    # Keep stdout for the one JSON line: anything else written to fd 1
    # (NCCL's version banner, library chatter) goes to stderr.
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse()
    from rustcompute_b200 import configs
    _, world, _ = dist_env()
    if args.scaling is None:
        args.scaling = "weak" if world > 1 else "strong"
    if args.grid:
        W, H, D = (int(v) for v in args.grid.lower().split("x"))
    else:
        base = configs.build(args.workload, steps=1)
        W, H, D = base.W, base.H, base.D
    if args.scaling == "weak" and world > 1:
        D *= world          # one D-plane slab per GPU
    wl = configs.build(args.workload, W, H, D)
    if args.impl == "reference":
        run_reference(args, wl)
        return
    run_ours(args, wl)


if __name__ == "__main__":
    main()
