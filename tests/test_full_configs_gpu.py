"""GPU parity at the benchmark configurations' (c1..c5) stated sizes and step counts.

Each case runs the path bench.py times -- variant auto through the C-ABI, which
takes the two-step kernel (k_step_tma2) for every pair of steps where it
applies -- on the full grid for the full step count, and compares the final
pressure and pressure_prev with

  * the CPU oracle (the C restatement of grid3d.rs:222-370, all host threads),
    run in a thread while the GPU computes: the north-star tolerance first
    (rel-L2 <= 1e-5, max|diff| <= 1e-4 * peak), then bit equality;
  * the SHA-256 digests in tests/golden/golden_full.json, made by
    tests/golden/make_golden.py --full from the same oracle.

  C2 256^3, 10 Ricker sources, sponge 16, 1000 steps
  C3 512^3 heterogeneous (8 layers + 32 spheres), sponge 16, 1 source, 500 steps
  C4 1024^3 layered, sponge 16, 1 source, 200 steps
  C5 128^3 Gaussian, 10,000 steps: per-step launches, and all 10,000 steps in
     one persistent (cooperative) launch
C1 at its full size is in test_parity_gpu.py.  Semantics: grid3d.rs:222-269.
"""
import hashlib
import json
import os
import threading

import numpy as np
import pytest

import oracle
from rustcompute_b200 import GpuBackend3D, configs

pytestmark = pytest.mark.gpu

REL_L2 = 1e-5
MAX_ABS_FRAC = 1e-4
HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "golden_full.json")) as _fh:
    GOLDEN = json.load(_fh)


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(memoryview(np.ascontiguousarray(a, np.float32)).cast("B")).hexdigest()


class OracleRun(threading.Thread):
    """The oracle on all host threads, in the background (the ctypes call
    releases the GIL, so the GPU run proceeds meanwhile)."""

    def __init__(self, wl):
        super().__init__(daemon=True)
        self.wl, self.grid, self.exc = wl, None, None
        self.start()

    def run(self):
        try:
            g = oracle.from_workload(self.wl)
            g.run(self.wl.steps, oracle.max_threads())
            self.grid = g
        except BaseException as e:  # reported by result()
            self.exc = e

    def result(self):
        self.join()
        if self.exc is not None:
            raise self.exc
        return self.grid


def assert_parity_chunked(got: np.ndarray, want: np.ndarray, what: str) -> None:
    """North-star tolerance, then bit equality, in chunks (1024^3 fields)."""
    assert got.shape == want.shape, what
    n, step = want.size, 1 << 25
    d2 = w2 = 0.0
    dmax = peak = 0.0
    for i in range(0, n, step):
        g = got[i:i + step].astype(np.float64)
        w = want[i:i + step].astype(np.float64)
        assert np.all(np.isfinite(g)), f"{what}: non-finite values near {i}"
        d = g - w
        d2 += float(np.dot(d, d))
        w2 += float(np.dot(w, w))
        dmax = max(dmax, float(np.max(np.abs(d))))
        peak = max(peak, float(np.max(np.abs(w))))
    rel = (d2 ** 0.5) / (w2 ** 0.5) if w2 > 0 else d2 ** 0.5
    assert rel <= REL_L2, f"{what}: rel-L2 {rel:.3e}"
    assert dmax <= MAX_ABS_FRAC * peak + 1e-30, f"{what}: max-abs {dmax:.3e} (peak {peak:.3e})"
    if not np.array_equal(got.view(np.uint32), want.view(np.uint32)):
        bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
        raise AssertionError(f"{what}: {bad.size} cells differ in bits, first at {bad[:5]} "
                             f"(rel-L2 {rel:.3e}, max-abs {dmax:.3e})")


def run_gpu(wl, mode: str):
    b = GpuBackend3D.create(wl.W, wl.H, wl.D, c_squared=wl.c_squared, damping=wl.damping,
                            sponge_width=wl.sponge_width, sponge_max=wl.sponge_max)
    p0, pp0 = wl.initial_fields()
    b.upload_fields(p0, pp0)
    del p0, pp0
    c2 = wl.c2_field()
    if c2 is not None:
        b.set_c2_field(c2)
    del c2
    if len(wl.sources):
        b.set_sources(wl.sources, wl.wavelet)
    if mode == "persistent":
        b.step_persistent(wl.steps)
    else:
        b.step_n(None, wl.steps)
    b.sync()
    stats = b.stats()
    p, pp = b.download_field(with_prev=True)
    b.close()
    return p, pp, stats


CASES = [
    ("c2_full", "c2", "step"),
    ("c3_full", "c3", "step"),
    ("c4_full", "c4", "step"),
    ("c5_full", "c5", "step"),
    ("c5_full", "c5", "persistent"),
]


@pytest.mark.parametrize("key,name,mode", CASES, ids=[f"{c[1]}-{c[2]}" for c in CASES])
def test_full_config_matches_oracle_and_golden(key, name, mode):
    wl = configs.build(name)
    gold = GOLDEN[key]
    assert gold["grid"] == [wl.W, wl.H, wl.D] and gold["steps"] == wl.steps
    ref = OracleRun(wl)
    p, pp, st = run_gpu(wl, mode)
    assert st["step"] == wl.steps
    if mode == "step" and wl.W > 128:
        # the kernel bench.py times: every pair of steps in one two-step launch
        assert st["two_step_launches"] == wl.steps // 2, st
    assert float(np.max(np.abs(p))) > 1e-6
    g = ref.result()
    assert_parity_chunked(p, g.pressure, f"{key}/{mode}/pressure")
    assert_parity_chunked(pp, g.pressure_prev, f"{key}/{mode}/pressure_prev")
    assert digest(p) == gold["sha256_pressure"], f"{key}/{mode}: pressure digest"
    assert digest(pp) == gold["sha256_pressure_prev"], f"{key}/{mode}: pressure_prev digest"
