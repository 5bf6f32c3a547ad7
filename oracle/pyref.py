"""Pure-Python restatement of the reference step, for tiny grids only.

TEST INFRASTRUCTURE ONLY.  An independent second restatement of
crates/ringkernel-wavesim3d/src/simulation/grid3d.rs:222-269 and :353-370,
written with numpy float32 scalars in the reference operation order, used to
cross-check the C oracle bit for bit.  Cost is O(cells) Python operations
per step, so keep grids to a few thousand cells.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def step(W, H, D, p, pp, c2=0.25, damping=1.0, types=None, refl=None, c2_field=None,
         sponge=None):
    """One step; returns the new (pressure, pressure_prev) pair (swapped)."""
    p = np.asarray(p, dtype=np.float32)
    out = np.array(pp, dtype=np.float32, copy=True)
    S = W * H
    c2s, damp = f32(c2), f32(damping)
    six, two = f32(6.0), f32(2.0)
    for z in range(1, D - 1):
        for y in range(1, H - 1):
            for x in range(1, W - 1):
                i = z * S + y * W + x
                if types is not None and types[i] != 0:
                    continue
                c = p[i]
                lap = f32(f32(f32(f32(f32(p[i - 1] + p[i + 1]) + p[i - W]) + p[i + W])
                              + p[i - S]) + p[i + S])
                lap = f32(lap - f32(six * c))
                cc = c2s if c2_field is None else f32(c2_field[i])
                pn = f32(f32(f32(two * c) - out[i]) + f32(cc * lap))
                v = f32(pn * damp)
                if sponge is not None and len(sponge):
                    d = min(x, W - 1 - x, y, H - 1 - y, z, D - 1 - z)
                    if d < len(sponge):
                        v = f32(v * f32(sponge[d]))
                out[i] = v
    for z in range(D):
        for y in range(H):
            for x in range(W):
                i = z * S + y * W + x
                if types is None:
                    face = x in (0, W - 1) or y in (0, H - 1) or z in (0, D - 1)
                    if face:
                        out[i] = f32(out[i] * f32(0.1))
                elif types[i] in (1, 3):
                    out[i] = f32(out[i] * f32(refl[i]))
    return out, p.copy()
