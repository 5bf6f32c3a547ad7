"""Regenerate the golden fixtures in this directory from the CPU oracle.

    python tests/golden/make_golden.py          # golden.json, slices, ragged case
    python tests/golden/make_golden.py --full   # golden_full.json (minutes, ~40 GB RAM)

The reference ships no field dumps for this path (its tests check only
qualitative properties), and its Rust crate cannot be built in this image, so
the fixtures are produced by the pinned C restatement in oracle/.  Each case
stores SHA-256 digests of the final pressure / pressure_prev bytes plus energy
and peak; the C1 case also stores its three centre slices, and one ragged case
stores its whole fields.

`--full` runs the five benchmark configurations (c1..c5) at their stated sizes and step
counts (C2 256^3 x 1000, C3 512^3 x 500, C4 1024^3 x 200, C5 128^3 x 10,000;
C1 is in golden.json already) on all host threads and stores the same digests
in golden_full.json.  tests/test_full_configs_gpu.py checks the CUDA path
against them and, in the same run, against the oracle on the GPU box's cores.
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from rustcompute_b200 import configs  # noqa: E402
from rustcompute_b200.grid import AcousticParams3D  # noqa: E402


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


def ragged_case():
    """13x7x5, seeded random fields, per-cell c2, sponge 2, 7 steps."""
    W, H, D = 13, 7, 5
    rng = np.random.default_rng(20261201)
    n = W * H * D
    c2 = rng.uniform(0.01, 0.25, n).astype(np.float32)
    g = oracle.OracleGrid(W, H, D, AcousticParams3D(c_squared=0.2, simple_damping=0.9995),
                          c2_field=c2, sponge_width=2, sponge_max=0.1)
    p0 = rng.standard_normal(n).astype(np.float32)
    pp0 = rng.standard_normal(n).astype(np.float32)
    g.pressure[:], g.pressure_prev[:] = p0, pp0
    g.run(7, 1)
    return dict(W=W, H=H, D=D, c2=c2, p0=p0, pp0=pp0, p=g.pressure.copy(),
                pp=g.pressure_prev.copy())


CASES = [
    ("c1_64x64x64_200", "c1", None),
    ("c2_40x36x34_60", "c2", (40, 36, 34, 60)),
    ("c3_96x72x64_90", "c3", (96, 72, 64, 90)),
    ("c4_64x64x48_40", "c4", (64, 64, 48, 40)),
    ("c5_48x48x48_300", "c5", (48, 48, 48, 300)),
    ("c3_160x64x40_40", "c3", (160, 64, 40, 40)),    # wide enough for the TMA kernel
    ("c2_144x40x36_50", "c2", (144, 40, 36, 50)),
]


def workload(name, dims):
    if dims is None:
        return configs.build(name)
    W, H, D, steps = dims
    return configs.build(name, W, H, D, steps=steps)


FULL_CASES = [
    ("c2_full", "c2"),
    ("c3_full", "c3"),
    ("c4_full", "c4"),
    ("c5_full", "c5"),
]


def full_main():
    import time
    path = os.path.join(HERE, "golden_full.json")
    out = {}
    if os.path.exists(path):
        with open(path) as fh:
            out = json.load(fh)
    only = [a for a in sys.argv[1:] if not a.startswith("--")]
    for key, name in FULL_CASES:
        if only and key not in only:
            continue
        wl = configs.build(name)
        t0 = time.perf_counter()
        g = oracle.from_workload(wl)
        g.run(wl.steps, oracle.max_threads())
        out[key] = {"workload": name, "grid": [wl.W, wl.H, wl.D], "steps": wl.steps,
                    "sha256_pressure": digest(g.pressure),
                    "sha256_pressure_prev": digest(g.pressure_prev),
                    "energy": float(np.dot(g.pressure.astype(np.float64),
                                           g.pressure.astype(np.float64))),
                    "max_pressure": float(np.max(np.abs(g.pressure)))}
        print(key, f"{time.perf_counter() - t0:.1f} s", json.dumps(out[key]), flush=True)
        del g
        with open(path, "w") as fh:
            json.dump(out, fh, indent=1, sort_keys=True)


def main():
    if "--full" in sys.argv:
        full_main()
        return
    out = {}
    for key, name, dims in CASES:
        wl = workload(name, dims)
        g = oracle.from_workload(wl)
        g.run(wl.steps, 1)
        out[key] = {"workload": name, "grid": [wl.W, wl.H, wl.D], "steps": wl.steps,
                    "sha256_pressure": digest(g.pressure),
                    "sha256_pressure_prev": digest(g.pressure_prev),
                    "energy": g.total_energy(), "max_pressure": g.max_pressure()}
        if key.startswith("c1_"):
            f = g.pressure.reshape(wl.D, wl.H, wl.W)
            np.savez_compressed(os.path.join(HERE, "c1_center_slices.npz"),
                                xy=f[wl.D // 2], xz=f[:, wl.H // 2, :], yz=f[:, :, wl.W // 2])
    r = ragged_case()
    np.savez_compressed(os.path.join(HERE, "ragged_13x7x5.npz"), **r)
    out["ragged_13x7x5_7"] = {"sha256_pressure": digest(r["p"]),
                              "sha256_pressure_prev": digest(r["pp"])}
    with open(os.path.join(HERE, "golden.json"), "w") as fh:
        json.dump(out, fh, indent=1, sort_keys=True)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
