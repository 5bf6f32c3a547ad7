"""Headless volume ray-march (visualization/volume.rs:76-160, :396-420).

CPU: the oracle's f16 quantiser equals IEEE round-to-nearest-even (numpy's
float16) over normal, subnormal and tie values; a known-answer image (a
uniform field seen head-on composites to (2, 0, 0, 2) exactly where rays hit
the box, as the shader's first sample already passes alpha 0.95); an empty
field is fully transparent; write_ppm's header and size.
GPU: the CUDA renderer equals the CPU restatement bit for bit (default
camera, explicit cameras inside and outside the box, compositing over a
background, a field after FDTD steps), and a z-slab context is refused.
"""
import os

import numpy as np
import pytest

import oracle
from rustcompute_b200.image import write_ppm


def smooth_field(W, H, D, seed=0):
    rng = np.random.default_rng(seed)
    f = rng.standard_normal((D, H, W)).astype(np.float32)
    for ax in range(3):   # a few box filters: smooth, signed values
        for _ in range(3):
            f = (np.roll(f, 1, ax) + f + np.roll(f, -1, ax)) / np.float32(3)
    return f.astype(np.float32)


def test_quantiser_is_round_to_nearest_even():
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.uniform(-1, 1, 20000), rng.uniform(-1e-4, 1e-4, 5000),
                        rng.uniform(-1e-7, 1e-7, 5000),
                        # exact ties between neighbouring halves
                        (np.arange(1, 200) + 0.5) * 2.0 ** -24,
                        1.0 + (np.arange(0, 64) + 0.5) * 2.0 ** -10,
                        [0.0, -0.0, 1.0, -1.0, 65504.0]]).astype(np.float32)
    want = x.astype(np.float16).astype(np.float32)
    got = oracle.quantize_f16(x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_known_answer_uniform_field_head_on():
    W = H = D = 8
    p = np.full((D, H, W), 0.5, np.float32)     # normalised to 1.0 everywhere
    img = oracle.render_volume(p, W, H, D, 32, 32, eye=(4, 4, 40), target=(4, 4, 4),
                               fov_y=0.5)
    hit = img[..., 3] > 0
    assert hit.any() and not hit.all()
    assert np.all(img[hit] == np.array([2.0, 0.0, 0.0, 2.0], np.float32))
    assert np.all(img[~hit] == 0.0)
    # the box covers the central pixels symmetrically
    assert np.array_equal(hit, hit[::-1, ::-1])


def test_empty_field_is_transparent():
    z = np.zeros((6, 7, 9), np.float32)
    img = oracle.render_volume(z, 9, 7, 6, 20, 10)
    assert not img.any()


def test_write_ppm(tmp_path):
    img = np.zeros((3, 5, 4), np.float32)
    img[1, 2] = (1.0, 0.5, 0.0, 1.0)
    path = os.path.join(tmp_path, "v.ppm")
    write_ppm(path, img)
    data = open(path, "rb").read()
    assert data.startswith(b"P6\n5 3\n255\n") and len(data) == len(b"P6\n5 3\n255\n") + 45
    px = data[len(b"P6\n5 3\n255\n"):]
    assert px[(1 * 5 + 2) * 3:(1 * 5 + 2) * 3 + 3] == bytes([255, 128, 0])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["default", "inside", "composite", "wide"])
def test_gpu_render_equals_cpu_restatement(case):
    from rustcompute_b200 import GpuBackend3D, SimulationGrid3D
    from rustcompute_b200.grid import AcousticParams3D
    W, H, D = 40, 24, 32
    f = smooth_field(W, H, D)
    g = SimulationGrid3D(W, H, D, AcousticParams3D(c_squared=0.25, simple_damping=1.0))
    g.pressure[:] = f.reshape(-1)
    g.pressure_prev[:] = f.reshape(-1)
    b = GpuBackend3D(g)
    kw = dict(default=dict(),
              inside=dict(eye=(20.5, 11.0, 15.0), target=(5.0, 3.0, 30.0), fov_y=1.0,
                          threshold=0.0, step_size=0.37, max_steps=50),
              composite=dict(cell_size=0.5, background=(0.1, 0.2, 0.3, 1.0), density_scale=0.7),
              wide=dict(eye=(-30.0, 50.0, -20.0), target=(20.0, 12.0, 16.0), up=(0.0, 0.0, 1.0),
                        fov_y=1.2, step_size=0.21))[case]
    w, h = (96, 54) if case != "wide" else (120, 40)
    got = b.render_volume(w, h, **kw)
    want = oracle.render_volume(f, W, H, D, w, h, **kw)
    assert (want[..., 3] > 0).mean() > 0.05          # the image shows something
    bad = np.flatnonzero(got.view(np.uint32) != want.view(np.uint32))
    assert bad.size == 0, f"{bad.size} values differ, first {bad[:4]}"
    b.close()


@pytest.mark.gpu
def test_gpu_render_after_steps_and_slab_refused():
    from rustcompute_b200 import GpuBackend3D, InvalidArgument, configs
    wl = configs.build("c1", 48, 40, 36, steps=30)
    b = GpuBackend3D.create(wl.W, wl.H, wl.D, c_squared=wl.c_squared, damping=wl.damping)
    p, pp = wl.initial_fields()
    b.upload_fields(p, pp)
    b.step_n(None, 30)
    field = b.download_field()
    got = b.render_volume(80, 60, threshold=0.005)
    want = oracle.render_volume(field, wl.W, wl.H, wl.D, 80, 60, threshold=0.005)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    b.close()
    s = GpuBackend3D.create(48, 40, 36, z_begin=0, z_end=18)
    with pytest.raises(InvalidArgument):
        s.render_volume(16, 16)
    s.close()
