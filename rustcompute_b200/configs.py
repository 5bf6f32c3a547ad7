"""Seeded synthetic workloads C1..C5 for the WaveSim3D FDTD step.

No public dataset is involved: every input is generated here from a seeded
SplitMix64 stream.  Floats drawn from the stream are (u64 >> 40) * 2^-24.
Transcendentals (Gaussian pulse, Ricker wavelet) and the medium are evaluated
in float64 and rounded once to float32, so the CUDA path and the CPU oracle
consume bit-identical inputs.

Configurations (the reference quotes only C1's shape; C2-C5 use features the
reference CPU path never had: per-cell speed, sponge, Ricker sources):
  C1  64^3, Courant^2 0.25, damping 1, Gaussian amp 1 sigma 3 at the centre in
      both fields, 200 steps, reference faces (absorber, reflection 0.1)
  C2  256^3, uniform, 10 Ricker sources >= 17 cells from the faces, sponge
      16 / 0.1, 1000 steps
  C3  512^3, 8 seeded z-layers + 32 seeded spheres (radius 10-40), speed
      ratio r in [0.3, 1], Courant^2 = (0.5 r)^2, sponge 16 / 0.1, one centred
      Ricker source, 500 steps
  C4  1024^3 layered (8 seeded layers), sponge 16 / 0.1, one centred Ricker
      source, 200 steps
  C5  128^3 uniform, Gaussian sigma 4, 10,000 steps (persistent mode)
Ricker: r(t) = (1 - 2 pi^2 f^2 tau^2) exp(-pi^2 f^2 tau^2), tau = t - 1.5/f,
f = 1/(40 dt) (20 cells per wavelength at Courant 0.5), t = step * dt, so
f*tau = (step - 60) / 40.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

MASK64 = (1 << 64) - 1


class SplitMix64:
    def __init__(self, seed: int):
        self.state = seed & MASK64

    def next_u64(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & MASK64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
        return z ^ (z >> 31)

    def uniform(self) -> float:
        """[0, 1) with 24 random bits."""
        return (self.next_u64() >> 40) * (1.0 / (1 << 24))

    def below(self, n: int) -> int:
        return self.next_u64() % n


def ricker(steps: int, delay_steps: float = 60.0, steps_per_period: float = 40.0) -> np.ndarray:
    s = np.arange(steps, dtype=np.float64)
    u = (s - delay_steps) / steps_per_period
    a = (math.pi ** 2) * u * u
    return ((1.0 - 2.0 * a) * np.exp(-a)).astype(np.float32)


def gaussian_field(W: int, H: int, D: int, cx: float, cy: float, cz: float, sigma: float,
                   amp: float = 1.0, z_begin: int = 0, z_end: Optional[int] = None) -> np.ndarray:
    z_end = D if z_end is None else z_end
    z = np.arange(z_begin, z_end, dtype=np.float64)[:, None, None]
    y = np.arange(H, dtype=np.float64)[None, :, None]
    x = np.arange(W, dtype=np.float64)[None, None, :]
    r2 = (x - cx) ** 2 + (y - cy) ** 2 + (z - cz) ** 2
    return (amp * np.exp(-r2 / (2.0 * sigma * sigma))).astype(np.float32).reshape(-1)


@dataclass
class Medium:
    """Piecewise-constant speed ratio: z-layers, then spheres painted over them."""

    layer_bounds: list          # len L+1, z boundaries (global)
    layer_r: list               # len L
    spheres: list = field(default_factory=list)   # (cx, cy, cz, radius, r)

    def c2_slab(self, W: int, H: int, z_begin: int, z_end: int) -> np.ndarray:
        """Courant^2 = (0.5 r)^2 for planes [z_begin, z_end), as a flat f32 array."""
        nz = z_end - z_begin
        r = np.empty((nz, H, W), dtype=np.float64)
        for (zb, ze), v in zip(zip(self.layer_bounds[:-1], self.layer_bounds[1:]), self.layer_r):
            a, b = max(zb, z_begin), min(ze, z_end)
            if a < b:
                r[a - z_begin:b - z_begin] = v
        for cx, cy, cz, rad, v in self.spheres:
            z0, z1 = max(int(math.floor(cz - rad)), z_begin), min(int(math.ceil(cz + rad)) + 1, z_end)
            if z0 >= z1:
                continue
            y0, y1 = max(int(math.floor(cy - rad)), 0), min(int(math.ceil(cy + rad)) + 1, H)
            x0, x1 = max(int(math.floor(cx - rad)), 0), min(int(math.ceil(cx + rad)) + 1, W)
            zz = np.arange(z0, z1, dtype=np.float64)[:, None, None]
            yy = np.arange(y0, y1, dtype=np.float64)[None, :, None]
            xx = np.arange(x0, x1, dtype=np.float64)[None, None, :]
            inside = (xx - cx) ** 2 + (yy - cy) ** 2 + (zz - cz) ** 2 <= rad * rad
            sub = r[z0 - z_begin:z1 - z_begin, y0:y1, x0:x1]
            sub[inside] = v
        return ((0.5 * r) ** 2).astype(np.float32).reshape(-1)


def seeded_medium(W: int, H: int, D: int, seed: int, n_layers: int = 8, n_spheres: int = 32,
                  r_lo: float = 0.3, r_hi: float = 1.0, rad_lo: float = 10.0,
                  rad_hi: float = 40.0) -> Medium:
    rng = SplitMix64(seed)
    cuts = sorted({1 + rng.below(max(D - 1, 1)) for _ in range(n_layers - 1)})
    while len(cuts) < n_layers - 1:  # extremely unlikely duplicate draw
        cuts = sorted(set(cuts) | {1 + rng.below(max(D - 1, 1))})
    bounds = [0] + cuts + [D]
    rs = [r_lo + (r_hi - r_lo) * rng.uniform() for _ in range(n_layers)]
    rs[rng.below(n_layers)] = r_hi  # c_max is reached somewhere: Courant 0.5 at c_max
    spheres = []
    for _ in range(n_spheres):
        cx, cy, cz = rng.below(W), rng.below(H), rng.below(D)
        rad = rad_lo + (rad_hi - rad_lo) * rng.uniform()
        v = r_lo + (r_hi - r_lo) * rng.uniform()
        spheres.append((float(cx), float(cy), float(cz), rad, v))
    return Medium(bounds, rs, spheres)


@dataclass
class Workload:
    name: str
    W: int
    H: int
    D: int
    steps: int
    c_squared: float = 0.25
    damping: float = 1.0
    sponge_width: int = 0
    sponge_max: float = 0.0
    gaussian: Optional[tuple] = None   # (cx, cy, cz, sigma, amp)
    medium: Optional[Medium] = None
    sources: np.ndarray = field(default_factory=lambda: np.zeros((0, 3), dtype=np.uint32))
    wavelet: np.ndarray = field(default_factory=lambda: np.zeros((0, 0), dtype=np.float32))

    @property
    def cells(self) -> int:
        return self.W * self.H * self.D

    @property
    def heterogeneous(self) -> bool:
        return self.medium is not None

    @property
    def bytes_per_cell_step(self) -> int:
        """Algorithmic HBM bytes: read p, read p_prev, write new (+ read c2)."""
        return 16 if self.heterogeneous else 12

    def initial_fields(self, z_begin: int = 0, z_end: Optional[int] = None):
        z_end = self.D if z_end is None else z_end
        n = (z_end - z_begin) * self.W * self.H
        if self.gaussian is None:
            p = np.zeros(n, dtype=np.float32)
        else:
            cx, cy, cz, sig, amp = self.gaussian
            p = gaussian_field(self.W, self.H, self.D, cx, cy, cz, sig, amp, z_begin, z_end)
        return p, p.copy()

    def c2_field(self, z_begin: int = 0, z_end: Optional[int] = None) -> Optional[np.ndarray]:
        if self.medium is None:
            return None
        z_end = self.D if z_end is None else z_end
        return self.medium.c2_slab(self.W, self.H, z_begin, z_end)

    def scaled(self, W: int, H: int, D: int, steps: Optional[int] = None) -> "Workload":
        """Same recipe at another size (for parity tests the oracle can finish)."""
        return build(self.name, W=W, H=H, D=D, steps=steps if steps is not None else self.steps)


def build(name: str, W: Optional[int] = None, H: Optional[int] = None, D: Optional[int] = None,
          steps: Optional[int] = None) -> Workload:
    name = name.lower()
    if name == "c1":
        W, H, D = W or 64, H or 64, D or 64
        return Workload("c1", W, H, D, steps if steps is not None else 200,
                        gaussian=(W // 2, H // 2, D // 2, 3.0, 1.0))
    if name == "c5":
        W, H, D = W or 128, H or 128, D or 128
        return Workload("c5", W, H, D, steps if steps is not None else 10000,
                        gaussian=(W // 2, H // 2, D // 2, 4.0, 1.0))
    if name == "c2":
        W, H, D = W or 256, H or 256, D or 256
        steps = steps if steps is not None else 1000
        rng = SplitMix64(0x5EED0002)
        margin = min(17, (min(W, H, D) - 1) // 2)
        pts = []
        for _ in range(10):
            pts.append([margin + rng.below(max(W - 2 * margin, 1)),
                        margin + rng.below(max(H - 2 * margin, 1)),
                        margin + rng.below(max(D - 2 * margin, 1))])
        wl = np.tile(ricker(steps), (10, 1))
        return Workload("c2", W, H, D, steps, sponge_width=min(16, (min(W, H, D) - 1) // 2),
                        sponge_max=0.1, sources=np.array(pts, dtype=np.uint32), wavelet=wl)
    if name in ("c3", "c4"):
        big = name == "c4"
        W, H, D = W or (1024 if big else 512), H or (1024 if big else 512), D or (1024 if big else 512)
        steps = steps if steps is not None else (200 if big else 500)
        seed = 0x5EED0004 if big else 0x5EED0003
        scale = min(W, H, D) / (1024.0 if big else 512.0)
        medium = seeded_medium(W, H, D, seed, n_layers=8, n_spheres=0 if big else 32,
                               rad_lo=max(10.0 * scale, 1.0), rad_hi=max(40.0 * scale, 2.0))
        src = np.array([[W // 2, H // 2, D // 2]], dtype=np.uint32)
        return Workload(name, W, H, D, steps, sponge_width=min(16, (min(W, H, D) - 1) // 2),
                        sponge_max=0.1, medium=medium, sources=src,
                        wavelet=ricker(steps)[None, :])
    raise ValueError(f"unknown workload {name!r}")
