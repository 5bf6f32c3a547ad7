"""Committed golden fixtures (tests/golden/, made by make_golden.py).

CPU: the oracle still reproduces every fixture bit for bit.
GPU: the CUDA step, through the C-ABI, reproduces them bit for bit.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import oracle
from rustcompute_b200 import GpuBackend3D, SimulationGrid3D, configs
from rustcompute_b200.grid import AcousticParams3D

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GOLD = json.load(open(os.path.join(HERE, "golden.json")))
CASES = [k for k in GOLD if not k.startswith("ragged")]


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


def workload(key):
    g = GOLD[key]
    W, H, D = g["grid"]
    return configs.build(g["workload"], W, H, D, steps=g["steps"])


@pytest.mark.parametrize("key", CASES)
def test_oracle_reproduces_golden(key):
    wl = workload(key)
    g = oracle.from_workload(wl)
    g.run(wl.steps, 1)
    assert digest(g.pressure) == GOLD[key]["sha256_pressure"]
    assert digest(g.pressure_prev) == GOLD[key]["sha256_pressure_prev"]


def test_oracle_reproduces_ragged_fixture():
    r = np.load(os.path.join(HERE, "ragged_13x7x5.npz"))
    W, H, D = int(r["W"]), int(r["H"]), int(r["D"])
    g = oracle.OracleGrid(W, H, D, AcousticParams3D(c_squared=0.2, simple_damping=0.9995),
                          c2_field=r["c2"], sponge_width=2, sponge_max=0.1)
    g.pressure[:], g.pressure_prev[:] = r["p0"], r["pp0"]
    g.run(7, 1)
    assert np.array_equal(g.pressure, r["p"]) and np.array_equal(g.pressure_prev, r["pp"])


def test_c1_slices_fixture_consistent():
    s = np.load(os.path.join(HERE, "c1_center_slices.npz"))
    assert s["xy"].shape == (64, 64) and float(np.max(np.abs(s["xy"]))) > 0


@pytest.mark.gpu
@pytest.mark.parametrize("variant", ["auto", "zstream", "naive", "refshape", "tma", "async", "tma2"])
@pytest.mark.parametrize("key", CASES)
def test_gpu_reproduces_golden(key, variant):
    wl = workload(key)
    if variant in ("tma", "tma2") and not (wl.W > 128 and wl.H >= 16):
        pytest.skip("TMA kernel needs W > 128 and H >= 16")
    g = SimulationGrid3D(wl.W, wl.H, wl.D,
                         AcousticParams3D(c_squared=wl.c_squared, simple_damping=wl.damping))
    g.pressure[:], g.pressure_prev[:] = wl.initial_fields()
    b = GpuBackend3D(g, variant=variant, sponge_width=wl.sponge_width, sponge_max=wl.sponge_max)
    c2 = wl.c2_field()
    if c2 is not None:
        b.set_c2_field(c2)
    if len(wl.sources):
        b.set_sources(wl.sources, wl.wavelet)
    b.step_n(g, wl.steps)
    b.download_pressure(g, with_prev=True)
    assert digest(g.pressure) == GOLD[key]["sha256_pressure"]
    assert digest(g.pressure_prev) == GOLD[key]["sha256_pressure_prev"]
    if key.startswith("c1_"):
        s = np.load(os.path.join(HERE, "c1_center_slices.npz"))
        f = g.pressure.reshape(wl.D, wl.H, wl.W)
        assert np.array_equal(f[wl.D // 2], s["xy"])


@pytest.mark.gpu
def test_gpu_reproduces_ragged_fixture():
    r = np.load(os.path.join(HERE, "ragged_13x7x5.npz"))
    W, H, D = int(r["W"]), int(r["H"]), int(r["D"])
    g = SimulationGrid3D(W, H, D, AcousticParams3D(c_squared=0.2, simple_damping=0.9995))
    g.pressure[:], g.pressure_prev[:] = r["p0"], r["pp0"]
    b = GpuBackend3D(g, sponge_width=2, sponge_max=0.1)
    b.set_c2_field(r["c2"])
    b.step_n(g, 7)
    b.download_pressure(g, with_prev=True)
    assert np.array_equal(g.pressure, r["p"]) and np.array_equal(g.pressure_prev, r["pp"])
