"""Two steps per launch (variant "tma2", temporal blocking) on the GPU.

One launch computes p_{t+1} and p_{t+2}; sources of step t+1 are applied
inside the launch.  Bar: bit-identical to the one-step TMA kernel (itself
bit-identical to the oracle) for every shape class the kernel sees -- tile and
chunk edges in x, y and z, ragged sizes, c2 fields, sponges, sources on tile
borders and coinciding sources, wavelets that end mid-launch, impulses
between calls, odd step counts -- and to the CPU oracle directly on a small
case.
"""
import numpy as np
import pytest

import oracle
from rustcompute_b200 import GpuBackend3D, _ffi, configs
from rustcompute_b200.grid import AcousticParams3D

pytestmark = pytest.mark.gpu


def make(W, H, D, variant, *, c2=None, sponge=0, sources=None, wavelet=None, seed=0,
         c_squared=0.2, damping=0.9995):
    rng = np.random.default_rng(seed)
    b = GpuBackend3D.create(W, H, D, c_squared=c_squared, damping=damping, variant=variant,
                            sponge_width=sponge, sponge_max=0.1)
    n = W * H * D
    b.upload_fields(rng.standard_normal(n).astype(np.float32),
                    rng.standard_normal(n).astype(np.float32))
    if c2 is not None:
        b.set_c2_field(c2)
    if sources is not None:
        b.set_sources(sources, wavelet)
    return b


def same_bits(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


def edge_sources(W, H, D, n, rng):
    """Sources on tile borders (x = 127/128/129, y = 7/8/9, ...), the grid
    faces, z-chunk borders, plus two coinciding pairs."""
    xs = [1, 2, 126, 127, 128, 129, 130, 255, 256, 257, W - 2, W - 1]
    ys = [1, 7, 8, 9, 15, 16, 17, 31, 32, 33, H - 2, H - 1]
    zs = [0, 1, 2, D // 2, D // 2 + 1, D - 2, D - 1]
    pts = [[xs[k % len(xs)] % W, ys[(3 * k) % len(ys)] % H, zs[(5 * k) % len(zs)] % D]
           for k in range(n - 2)]
    pts += [pts[0], pts[3]]          # coinciding sources add in order
    return np.array(pts, np.uint32), rng.standard_normal((n, 9)).astype(np.float32)


@pytest.mark.parametrize("shape", [(256, 32, 40), (300, 40, 33), (129, 20, 3), (160, 24, 1),
                                   (160, 24, 2), (520, 21, 12), (384, 72, 100), (200, 37, 9),
                                   (264, 50, 21)])
@pytest.mark.parametrize("c2f,sponge", [(False, 0), (True, 3)])
@pytest.mark.parametrize("steps", [2, 7, 12])
def test_two_step_equals_one_step(shape, c2f, sponge, steps):
    W, H, D = shape
    rng = np.random.default_rng(W + H + D)
    c2 = rng.uniform(0.01, 0.25, W * H * D).astype(np.float32) if c2f else None
    sw = min(sponge, max((min(shape) - 1) // 2, 0))
    src, wav = edge_sources(W, H, D, 12, rng)
    one = make(W, H, D, "tma", c2=c2, sponge=sw, sources=src, wavelet=wav, seed=D)
    two = make(W, H, D, "tma2", c2=c2, sponge=sw, sources=src, wavelet=wav, seed=D)
    one.step_n(None, steps)
    two.step_n(None, steps)
    p1, pp1 = one.download_field(with_prev=True)
    p2, pp2 = two.download_field(with_prev=True)
    assert same_bits(p2, p1), f"pressure differs in {(p1 != p2).sum()} cells"
    assert same_bits(pp2, pp1), f"pressure_prev differs in {(pp1 != pp2).sum()} cells"
    assert two.stats()["step"] == steps
    if H >= _ffi.WS3D_TWO_STEP_ROWS + 4:   # the two-step kernel's boxes fit: it ran
        assert two.stats()["two_step_launches"] == steps // 2
    one.close()
    two.close()


@pytest.mark.parametrize("stages", ["4", "5", None])
@pytest.mark.parametrize("shape", [(520, 21, 12), (384, 72, 100), (768, 24, 10), (1024, 26, 9)])
def test_both_pipeline_depths_equal_one_step(monkeypatch, stages, shape):
    """The two-step kernel has a 4- and a 5-stage TMA pipeline (chosen by row
    size, 5 while a field takes at most 1.5 GiB; WS3D_TWO_STEP_STAGES at create
    forces one):
    both equal single steps bit for bit, with a c2 field, a sponge and edge
    sources."""
    if stages is None:
        monkeypatch.delenv("WS3D_TWO_STEP_STAGES", raising=False)
    else:
        monkeypatch.setenv("WS3D_TWO_STEP_STAGES", stages)
    W, H, D = shape
    rng = np.random.default_rng(W * 7 + D)
    c2 = rng.uniform(0.01, 0.25, W * H * D).astype(np.float32)
    src, wav = edge_sources(W, H, D, 12, rng)
    one = make(W, H, D, "tma", c2=c2, sponge=3, sources=src, wavelet=wav, seed=D)
    two = make(W, H, D, "tma2", c2=c2, sponge=3, sources=src, wavelet=wav, seed=D)
    one.step_n(None, 9)
    two.step_n(None, 9)
    p1, pp1 = one.download_field(with_prev=True)
    p2, pp2 = two.download_field(with_prev=True)
    assert same_bits(p2, p1), f"pressure differs in {(p1 != p2).sum()} cells"
    assert same_bits(pp2, pp1), f"pressure_prev differs in {(pp1 != pp2).sum()} cells"
    assert two.stats()["two_step_launches"] == 4
    one.close()
    two.close()


def test_two_step_matches_oracle_with_sources():
    wl = configs.build("c2", 144, 40, 36, steps=30)
    ref = oracle.from_workload(wl)
    ref.run(wl.steps, 1)
    b = GpuBackend3D.create(wl.W, wl.H, wl.D, c_squared=wl.c_squared, damping=wl.damping,
                            variant="tma2", sponge_width=wl.sponge_width,
                            sponge_max=wl.sponge_max)
    p, pp = wl.initial_fields()
    b.upload_fields(p, pp)
    if wl.c2_field() is not None:
        b.set_c2_field(wl.c2_field())
    b.set_sources(wl.sources, wl.wavelet)
    b.step_n(None, wl.steps)
    gp, gpp = b.download_field(with_prev=True)
    assert float(np.max(np.abs(ref.pressure))) > 1e-4
    assert same_bits(gp, ref.pressure)
    assert same_bits(gpp, ref.pressure_prev)
    b.close()


def test_wavelet_ends_inside_a_launch_and_many_sources_fall_back():
    W, H, D = 200, 24, 20
    rng = np.random.default_rng(5)
    # wavelet of odd length: the launch covering steps (len-1, len) applies a
    # zero amplitude for step len, exactly like the one-step path
    src = np.array([[100, 12, 10], [128, 8, 9], [127, 7, 11]], np.uint32)
    wav = rng.standard_normal((3, 5)).astype(np.float32)
    one = make(W, H, D, "tma", sources=src, wavelet=wav)
    two = make(W, H, D, "tma2", sources=src, wavelet=wav)
    one.step_n(None, 10)
    two.step_n(None, 10)
    assert same_bits(two.download_field(), one.download_field())
    # 40 sources: more than the two-step kernel holds, so single TMA steps run
    src40 = np.stack([rng.integers(0, W, 40), rng.integers(0, H, 40), rng.integers(0, D, 40)],
                     1).astype(np.uint32)
    wav40 = rng.standard_normal((40, 8)).astype(np.float32)
    one.set_sources(src40, wav40)
    two.set_sources(src40, wav40)
    one.step_n(None, 6)
    two.step_n(None, 6)
    assert same_bits(two.download_field(), one.download_field())
    one.close()
    two.close()


def test_impulses_between_calls_and_split_calls():
    W, H, D = 256, 40, 48
    rng = np.random.default_rng(9)
    src, wav = edge_sources(W, H, D, 6, rng)
    one = make(W, H, D, "tma", sources=src, wavelet=wav)
    two = make(W, H, D, "tma2", sources=src, wavelet=wav)
    for n, imp in ((3, (128, 8, 0)), (4, (127, 16, 24)), (1, (5, 5, 47)), (6, (200, 39, 1))):
        for b in (one, two):
            b.step_n(None, n)
            b.inject_impulse(*imp, 0.75)
            b.inject_spherical_impulse(W // 2, H // 2, D // 2, 0.3, 2.5)
    p1, pp1 = one.download_field(with_prev=True)
    p2, pp2 = two.download_field(with_prev=True)
    assert same_bits(p2, p1) and same_bits(pp2, pp1)
    assert one.energy() == two.energy()
    one.close()
    two.close()


def test_two_step_memory_timing_and_launch_count():
    W, H, D = 256, 64, 64
    one = make(W, H, D, "tma")
    two = make(W, H, D, "tma2")
    # the two extra field buffers are allocated with the context, not in a step
    slab = 256 * 64 * (64 + 2) * 4
    assert two.memory_usage() - one.memory_usage() == 2 * slab
    before = two.memory_usage()
    l0 = two.stats()["kernel_launches"]
    ms = two.step_timed(10)       # 5 two-step launches
    assert ms > 0.0
    assert two.stats()["kernel_launches"] - l0 == 5
    assert two.memory_usage() == before
    one.close()
    two.step_n(None, 3)           # one two-step launch and one single step
    assert two.stats()["kernel_launches"] - l0 == 7
    assert two.stats()["step"] == 13
    two.close()
