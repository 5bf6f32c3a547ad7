"""bench.py's output contract, on CPU: the reference arm (the CPU step of the
path, restated in oracle/) prints one JSON line with the keys the driver
reads, and the roofline / kernel naming logic of our arm matches the library's
launch choices.  No GPU is touched.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def run_bench(*args):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.strip().splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = run_bench("--impl", "reference", "--grid", "96x64x40", "--steps", "2", "--warmup", "1")
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["unit"] == "Mcells/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "c3" and d["config"]["grid"] == [96, 64, 40]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_kernel_name_follows_the_library_choice():
    import bench
    from rustcompute_b200 import configs
    c3 = configs.build("c3", 512, 512, 512, steps=10)
    narrow = configs.build("c3", 96, 64, 64, steps=10)
    many = configs.build("c2", 256, 64, 64, steps=10)
    many.sources = many.sources.repeat(4, axis=0)          # 40 sources: over the two-step table
    assert bench.kernel_name("auto", c3, 1) == "k_step_tma2"
    assert bench.kernel_name("auto", c3, 2) == "k_step_tma"              # slabs at depth 1
    assert bench.kernel_name("auto", c3, 2, depth=2) == "k_step_tma2"    # slabs at depth 2
    assert bench.kernel_name("auto", narrow, 1) == "k_step_naive"        # boxes do not fit, small
    assert bench.kernel_name("auto", narrow, 2) == "k_step_zstream"      # z-slabs
    wide_narrow = configs.build("c3", 96, 512, 512, steps=10)
    assert bench.kernel_name("auto", wide_narrow, 1) == "k_step_zstream"
    assert bench.kernel_name("auto", many, 1) == "k_step_tma"
    assert bench.kernel_name("tma", c3, 1) == "k_step_tma"
    small = configs.build("c5", 128, 128, 128, steps=10)
    assert bench.kernel_name("auto", c3, 1, mode="persistent") == "k_persistent_rows"
    assert bench.kernel_name("auto", small, 1, mode="persistent") == "k_persistent_smem"
    assert bench.kernel_name("auto", small, 2, mode="persistent") == "k_persistent_rows"
    assert bench.kernel_name("auto", c3, 1, mode="resident") == "k_resident"


def test_cpu_legs_time_the_same_steps_from_the_initial_state():
    """cpu_baseline and the reference arm time steps W..W+K of the same sample;
    every cpu_baseline run restarts from the workload's initial state, so each
    run computes the same fields."""
    import numpy as np

    import bench
    from rustcompute_b200 import configs
    wl = configs.build("c3", 64, 48, 40, steps=12)
    sample, desc = bench.reference_sample(wl, 6, 3, 2)
    assert sample is wl and desc.startswith("full 64x48x40")
    r = bench.ReferenceCpuRun(sample, 2)
    v1, dt1 = r.run(6, 3)
    p1 = r.g.pressure.copy()
    v2, dt2 = r.run(6, 3)
    assert v1 > 0 and v2 > 0 and dt1 > 0 and dt2 > 0
    assert r.g.step == 9
    assert np.array_equal(p1.view(np.uint32), r.g.pressure.view(np.uint32))
    cb = bench.cpu_baseline_leg(wl, 6, 3, target_s=0.05, max_runs=3)
    assert cb["kind"] == "port" and cb["unit"] == "Mcells/s" and 1 <= cb["runs"] <= 3
    assert cb["min"] <= cb["value"] <= cb["max"]
    assert "steps 3..9" in cb["sample"] and cb["nproc"] >= 1
