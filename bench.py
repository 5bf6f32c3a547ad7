#!/usr/bin/env python
"""Benchmark of the B200 WaveSim3D FDTD step (configuration c3 by default).

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
                         "(grid W x H x D*N, as configuration c4's weak scaling); strong "
                         "splits the single-GPU grid into N slabs")
    ap.add_argument("--grid", default=None,
                    help="WxHxD: the workload's recipe at another size (profiling cases)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-c5", action="store_true",
                    help="skip the configuration c5 latency figures (persistent launch vs one "
                         "launch per step, 128^3) added to the line")
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


def ncu_traffic(wl, kernel: str, slab_planes: int = 0):
    """DRAM bytes per launch of the step kernel from a committed ncu summary
    (profiles/traffic.json, keyed by workload, grid and kernel; z-slabs by the
    slab's own size, `slab_planes` > 0), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    key = (f"{wl.name}/slab{wl.W}x{wl.H}x{slab_planes}/{kernel}" if slab_planes
           else f"{wl.name}/{wl.W}x{wl.H}x{wl.D}/{kernel}")
    e = d.get(key)
    return None if e is None else e.get("dram_bytes_per_launch")


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML (read-only)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device: int, period_s: float = 0.005):
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


def cpu_info() -> dict:
    """CPU model and core counts of this host (recorded beside the CPU figures)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count(), "threads_allowed": host_threads()}


def reference_sample(wl, steps: int, warmup: int, nthreads: int, budget_s: float = 150.0):
    """The grid the CPU legs time per step: the full grid when warmup + steps
    full-grid steps fit in about budget_s on this host, else a z-slab of the
    same recipe (same per-cell work)."""
    import oracle
    probe = wl.scaled(wl.W, wl.H, min(wl.D, 34), steps=4)
    g = oracle.from_workload(probe)
    g.run(2, nthreads)
    t0 = time.perf_counter()
    g.run(2, nthreads)
    rate = 2 * probe.cells / max(time.perf_counter() - t0, 1e-9)
    budget = budget_s / max(steps + warmup, 1)
    if wl.cells / rate <= budget:
        return wl, f"full {wl.W}x{wl.H}x{wl.D} grid per step"
    planes = max(8, min(wl.D, int(budget * rate / (wl.W * wl.H))))
    sample = wl.scaled(wl.W, wl.H, planes, steps=steps + warmup + 1)
    return sample, (f"{wl.W}x{wl.H}x{planes} z-slab of the {wl.name} recipe per step "
                    "(bounded sample)")


class ReferenceCpuRun:
    """Steps warmup .. warmup + steps of `sample` on the CPU restatement of the
    reference step (OpenMP over z-planes like step_parallel), from the
    workload's initial state every run.

    Both CPU legs time exactly these steps, because the CPU's cost per step
    depends on where the simulation is: the spreading wave front leaves
    subnormal values behind it (2.5 % of the cells of a 512 x 512 x 128 C3
    grid after 300 steps), and the host pays a microcode assist for each
    subnormal operand, so later steps run up to 2x slower (measured on the
    oracle: 1.08 Gcells/s at step 10, 0.55 at step 312, 8 threads).  The GPU
    handles subnormals at full rate."""

    def __init__(self, sample, nthreads: int):
        import oracle
        self.sample, self.nthreads = sample, nthreads
        self.g = oracle.from_workload(sample)
        self.p0 = self.g.pressure.copy()
        self.pp0 = self.g.pressure_prev.copy()

    def run(self, steps: int, warmup: int) -> tuple[float, float]:
        g = self.g
        g.pressure[:] = self.p0
        g.pressure_prev[:] = self.pp0
        g.step, g.time = 0, np.float32(0.0)
        g.run(warmup, self.nthreads)
        t0 = time.perf_counter()
        g.run(steps, self.nthreads)
        dt = time.perf_counter() - t0
        return self.sample.cells * steps / dt / 1e6, dt


def cpu_baseline_leg(wl, steps: int, warmup: int, target_s: float = 10.0,
                     max_runs: int = 25) -> dict:
    """The bench line's cpu_baseline (rank 0, N = 1): the same steps of the same
    sample as the reference arm (--impl reference), repeated from the initial
    state until about target_s of timed CPU work; the median run is reported."""
    nthreads = host_threads()
    sample, desc = reference_sample(wl, steps, warmup, nthreads)
    r = ReferenceCpuRun(sample, nthreads)
    rates, secs = [], 0.0
    while len(rates) < max_runs and (secs < target_s or not rates):
        v, dt = r.run(steps, warmup)
        rates.append(v)
        secs += dt
    return {"value": float(statistics.median(rates)), "unit": UNIT, "cores": nthreads,
            "kind": "port",
            "sample": f"{desc}; steps {warmup}..{warmup + steps} after {warmup} untimed steps "
                      f"(the steps the reference arm times), median of {len(rates)} runs from "
                      "the initial state",
            "seconds": secs, "runs": len(rates), "min": min(rates), "max": max(rates),
            **cpu_info()}


def run_reference(args, wl):
    """--impl reference: the reference's CPU path (C restatement) on host cores."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    nthreads = host_threads()
    warmup = max(args.warmup, 3)
    sample, desc = reference_sample(wl, args.steps, warmup, nthreads)
    val, dt = ReferenceCpuRun(sample, nthreads).run(args.steps, warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": warmup, "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SplitMix64 medium and sources)",
        "config": {"workload": wl.name, "grid": [wl.W, wl.H, wl.D],
                   "heterogeneous": wl.heterogeneous, "sponge": wl.sponge_width,
                   "sources": int(len(wl.sources))},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": f"{desc}; steps {warmup}..{warmup + args.steps} after "
                                   f"{warmup} untimed steps", **cpu_info()},
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
    if mode == "persistent":   # rows of at most 128 cells on one GPU: field in shared memory
        return "k_persistent_smem" if world == 1 and wl.W <= 128 else "k_persistent_rows"
    if mode == "resident":
        return "k_resident"
    if variant in ("auto", "tma2"):   # mirrors the library's choice for the default faces
        from rustcompute_b200 import _ffi
        tma_ok = wl.W > 128 and wl.H >= 16
        two_step = (world == 1 or depth == 2) and tma_ok and len(wl.sources) <= 32 and \
            wl.sponge_width <= 64 and wl.H >= _ffi.WS3D_TWO_STEP_ROWS + 4
        pitch = (wl.W + 31) // 32 * 32
        small = world == 1 and pitch * wl.H * wl.D * 4 <= 8 << 20   # one thread per cell
        variant = "tma2" if two_step else ("tma" if tma_ok else "naive" if small else "zstream")
    return {"tma": "k_step_tma", "tma2": "k_step_tma2", "async": "k_step_async",
            "zstream": "k_step_zstream",
            "naive": "k_step_naive", "refshape": "k_ref_stencil+k_ref_boundary"}[variant]


def plane_digests(field: np.ndarray, plane_cells: int) -> list:
    """SHA-256 of every z-plane of a flat f32 field."""
    import hashlib
    mv = memoryview(np.ascontiguousarray(field)).cast("B")
    step = plane_cells * 4
    return [hashlib.sha256(mv[i:i + step]).hexdigest() for i in range(0, len(mv), step)]


def slab_parity(b, wl, args, rank, world, local, pg, depth) -> dict:
    """N > 1, after the timed region: every rank's slab of the final field
    against ONE GPU (rank 0's) running the whole grid for the same number of
    steps through the same public API, compared plane by plane via SHA-256
    digests gathered over the process group (the reference checks its P2P
    transfers byte for byte the same way, with a CRC, multi_gpu/runtime.rs).
    One GPU's result equals the oracle bit for bit (tests/), so a match here
    is bit-exactness of the z-slab exchange at this N."""
    import torch
    steps = max(args.warmup, 3) + args.steps
    plane = wl.W * wl.H
    mine = plane_digests(b.download_field(), plane)
    gathered = [None] * world
    pg.all_gather_object(gathered, mine)
    out = {"reference": f"one GPU, whole {wl.W}x{wl.H}x{wl.D} grid, {steps} steps "
                        "(variant auto)", "steps": steps, "halo_depth": depth}
    # the whole grid on one GPU: five field-sized buffers (p, p_prev, two
    # two-step outputs, c2) beside this rank's own slab context, and about 24
    # host bytes per cell to build its inputs
    need = 5 * 4 * wl.cells
    free = torch.cuda.mem_get_info(local)[0] if rank == 0 else 0
    if rank == 0 and (need > 0.9 * free or wl.cells > (1 << 31)):
        out["result"] = "skipped"
        out["why"] = (f"the whole grid ({wl.cells} cells, {need / 2 ** 30:.1f} GiB on the device) "
                      "does not fit one GPU beside its slab")
    elif rank == 0:
        full = make_backend(wl, "auto", local, 0, wl.D)
        p, pp = wl.initial_fields()
        full.upload_fields(p, pp)
        del p, pp
        c2 = wl.c2_field()
        if c2 is not None:
            full.set_c2_field(c2)
        del c2
        if len(wl.sources):
            full.set_sources(wl.sources, wl.wavelet)
        full.step_n(None, steps)
        want = plane_digests(full.download_field(), plane)
        full.close()
        got = [d for r in range(world) for d in gathered[r]]
        bad = [z for z in range(wl.D) if got[z] != want[z]]
        out["result"] = "bit-exact" if not bad else "differs"
        if bad:
            out["first_differing_plane"] = bad[0]
            out["differing_planes"] = len(bad)
    pg.barrier()
    return out


def c5_latency(world, rank, local, pg, barrier, per_rank, stream, dev, device_gate) -> dict:
    """configuration c5 beside the main line: 128^3 uniform Gaussian on the same
    GPUs (z-slabs at N > 1, halos by in-kernel peer stores and flags), all
    10,000 steps in ONE persistent (cooperative) launch against one launch per
    step; microseconds per step, max over ranks, CUDA events on the launch
    stream after a device-side start gate."""
    import torch
    from rustcompute_b200 import configs
    wl5 = configs.build("c5")
    zb, ze = slab_bounds(wl5.D, world, rank)
    # zstream: one launch per step for the per-step leg (auto would run a
    # multi-step call on this small grid as one persistent launch too)
    b = make_backend(wl5, "zstream", local, zb, ze)
    b.set_stream(stream.cuda_stream)
    p, pp = wl5.initial_fields(zb, ze)
    b.upload_fields(p, pp)
    if world > 1:
        from rustcompute_b200.slab import connect
        connect(b, rank, world, pg.all_gather_object, barrier)

    def timed(fn) -> float:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        device_gate()
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return max(per_rank(e0.elapsed_time(e1)))

    b.step_n(None, 100)
    n_launch = 2000
    launch_ms = timed(lambda: b.step_n(None, n_launch))
    b.step_persistent(100)
    pers_ms = timed(lambda: b.step_persistent(wl5.steps))
    b.sync()
    b.close()
    return {"grid": [wl5.W, wl5.H, wl5.D], "n_gpus": world,
            "persistent_us_per_step": pers_ms * 1e3 / wl5.steps,
            "persistent_steps": wl5.steps,
            "launch_per_step_us_per_step": launch_ms * 1e3 / n_launch,
            "launch_per_step_steps": n_launch,
            "kernels": "one cooperative launch (k_persistent_smem on one GPU: the field in "
                       "shared memory, faces exchanged as step-tagged words; k_persistent_rows "
                       "on z-slabs: one grid barrier per step) vs one k_step_zstream launch per "
                       "step"}


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

    def per_rank(v: float) -> list:
        """v from every rank, in rank order (host plumbing only)."""
        if pg is None:
            return [v]
        t = torch.zeros(world, device=dev, dtype=torch.float64)
        t[rank] = v
        pg.all_reduce(t)
        return [float(x) for x in t.tolist()]

    stream = torch.cuda.Stream(device=dev)   # a real stream (handle != 0) shared with the library
    gate_t = torch.ones(1, device=dev)

    def device_gate():
        """N > 1: an all-reduce enqueued on the launch stream just before the
        start event.  The event then fires on every rank when the collective
        completes (within microseconds of each other), however far apart the
        host threads reached this point, so no rank's timed region starts by
        waiting for a neighbour that has not started yet."""
        if pg is not None:
            with torch.cuda.stream(stream):
                pg.all_reduce(gate_t)
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
    if world > 1:
        b.halo_wait_stats(reset=True)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        device_gate()
        host_start = time.time()
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
            # the end event goes right behind the last launch; the library's
            # per-launch events are summed after it
            b.step_timed_begin(args.steps)
            e1.record(stream)
            kernel_ms = b.step_timed_end()
        torch.cuda.synchronize(dev)
    barrier()
    launches = b.stats()["kernel_launches"] - launches0
    span_ms = per_rank(host_ms if args.mode == "resident" else e0.elapsed_time(e1))
    total_ms = max(span_ms)
    value = wl.cells * args.steps / (total_ms * 1e-3) / 1e6
    starts = per_rank(host_start)
    waits = b.halo_wait_stats() if world > 1 else (0, 0)
    wait_ns, wait_n = per_rank(float(waits[0])), per_rank(float(waits[1]))

    if kernel_ms is None:   # persistent / resident: the one launch is the whole timed region
        kernel_ms = span_ms[rank]
    kernel_ms_ranks = per_rank(kernel_ms)
    kernel_ms = max(kernel_ms_ranks)   # the slowest rank's kernels
    bpc = wl.bytes_per_cell_step
    kname = kernel_name(args.variant, wl, world, args.mode, depth)
    # auto on a small one-GPU grid runs the K steps as one persistent launch
    one_launch = args.mode == "step" and world == 1 and args.steps >= 2 and launches == 1
    if one_launch:
        kname = "k_persistent_smem"
    if one_launch:
        n_launch = 1
        total_bytes = bpc * local_cells * args.steps
        alg_bytes = total_bytes
    elif kname == "k_step_tma2" and args.mode == "step":
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
                "traffic": ncu_traffic(wl, kernel_name(args.variant, wl, world, depth=depth),
                                       ze - zb if world > 1 else 0),
                "algorithmic_bytes_per_launch": alg_bytes,
                "steps_per_launch": args.steps if one_launch else
                                    2 if kname == "k_step_tma2" and args.mode == "step" else 1,
                # algorithmic bytes per cell of one launch: one step moves bpc (read p,
                # p_prev (+ c2), write one field); a two-step launch bpc + 4 (one more write)
                "bytes_per_cell_per_launch": alg_bytes // max(local_cells, 1),
                "bytes_per_cell_step": bpc,
                "kernel_avg_ms": avg_kernel_ms,
                "kernel_avg_ms_per_rank": [v / n_launch for v in kernel_ms_ranks],
                "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"
                               if peaks["source"] == "measured" else "fallback",
                "kernel": kname,
                "ranks": "kernel_avg_ms and frac: the slowest rank (max over ranks)"}

    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded SplitMix64 medium and sources)",
        "config": {"workload": wl.name, "grid": [wl.W, wl.H, wl.D], "variant": args.variant,
                   "heterogeneous": wl.heterogeneous, "sponge": wl.sponge_width,
                   "sources": int(len(wl.sources)), "decomposition": f"z-slabs x{world}",
                   "halo_depth": depth,
                   "l2": ("inputs larger than L2 (each field %d MiB > 126 MB)"
                          if wl.cells * 4 > 126 * 10 ** 6 else
                          "fields L2-resident (each field %d MiB < 126 MB; no flush)")
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
    if world > 1:
        result["ranks"] = {
            "span_ms": span_ms,
            "halo_wait_ms": [v * 1e-6 for v in wait_ns],
            "halo_waits": [int(v) for v in wait_n],
            "host_start_skew_ms": (max(starts) - min(starts)) * 1e3,
            "start": "an all-reduce on the launch stream gates every rank's start event",
            "note": "span = the rank's start-to-end event time; halo_wait = device time its "
                    "step kernels spent in neighbour-flag waits that did not pass at once",
        }
        result["parity"] = slab_parity(b, wl, args, rank, world, local, pg, depth)
        # NVLink halo bytes per launch of an interior slab (two neighbours),
        # algorithmic: a two-step launch stores p_{t+2} of two edge planes into
        # each neighbour and reads the neighbour's p_{t-1} (and c2) edge plane;
        # a one-step launch stores one edge plane per neighbour
        plane_b = wl.W * wl.H * 4
        two = kname == "k_step_tma2" and args.mode == "step"
        per_nb = (2 + 1 + (1 if wl.heterogeneous else 0)) * plane_b if two else plane_b
        result["halo"] = {"nvlink_bytes_per_launch_interior_slab": 2 * per_nb,
                          "per_neighbour": {"stored": (2 if two else 1) * plane_b,
                                            "loaded": (per_nb - 2 * plane_b) if two else 0},
                          "steps_per_exchange": 2 if two else 1,
                          "note": "algorithmic; kernel peer stores and loads, no copies"}
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

    if not args.no_c5 and args.mode == "step":
        result["c5_latency"] = c5_latency(world, rank, local, pg, barrier, per_rank, stream, dev,
                                          device_gate)

    if rank == 0 and world == 1 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline_leg(wl, args.steps, max(args.warmup, 3))
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
