"""Writing rendered volumes to files (the headless stand-in for the
reference's window; visualization/renderer.rs presents to a surface)."""
from __future__ import annotations

import numpy as np


def write_ppm(path: str, rgba: np.ndarray) -> None:
    """Binary PPM (P6) of an RGBA float image in [0, 1]; alpha is dropped
    (composite over a background first to keep it)."""
    img = np.asarray(rgba, dtype=np.float32)
    if img.ndim != 3 or img.shape[2] < 3:
        raise ValueError("expected an (height, width, 4) image")
    rgb = (np.clip(img[:, :, :3], 0.0, 1.0) * 255.0 + 0.5).astype(np.uint8)
    h, w = rgb.shape[:2]
    with open(path, "wb") as f:
        f.write(b"P6\n%d %d\n255\n" % (w, h))
        f.write(rgb.tobytes())
