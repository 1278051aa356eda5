"""numpy restatement of the server's line-tensor construction (test oracle
only): write_line_tensor (server/src/lines.rs:98-135) with
write_rgb_tensor / write_resized_rgb_tensor (server/src/main.rs:1101-1150).

Rust rounds every float operation separately, as numpy float32 does, so this
restatement follows the reference operation for operation.
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


def natural_width(w: int, h: int) -> int:
    """ceil(48 * w / h), lines.rs:102."""
    if w <= 0 or h <= 0:
        raise ValueError("line dimensions must be positive")
    return -(-(w * 48) // h)


def line_tensor(img: np.ndarray, bucket: int) -> np.ndarray:
    """u8 [h, w, 3] -> f32 [3, 48, bucket] (lines.rs:115-135)."""
    h, w = img.shape[:2]
    rw = natural_width(w, h)
    if rw > bucket:
        raise ValueError(f"line normalized width {rw} exceeds maximum {bucket}; split the line crop")
    out = np.zeros((3, 48, bucket), f32)
    if w == rw and h == 48:
        v = img.astype(f32)
        out[:, :, :rw] = ((v / f32(255.0) - f32(0.5)) / f32(0.5)).transpose(2, 0, 1)
        return out
    sx_scale = f32(w) / f32(rw)
    sy_scale = f32(h) / f32(48)
    ys = np.arange(48, dtype=f32)
    xs = np.arange(rw, dtype=f32)
    sy = np.maximum((ys + f32(0.5)) * sy_scale - f32(0.5), f32(0.0)).astype(f32)
    sx = np.maximum((xs + f32(0.5)) * sx_scale - f32(0.5), f32(0.0)).astype(f32)
    y0 = np.minimum(np.floor(sy).astype(np.int64), h - 1)
    x0 = np.minimum(np.floor(sx).astype(np.int64), w - 1)
    y1 = np.minimum(y0 + 1, h - 1)
    x1 = np.minimum(x0 + 1, w - 1)
    wy = (sy - y0.astype(f32)).astype(f32)[:, None]
    wx = (sx - x0.astype(f32)).astype(f32)[None, :]
    one = f32(1.0)
    for c in range(3):
        p = img[..., c].astype(f32)
        top = (p[y0][:, x0] * (one - wx) + p[y0][:, x1] * wx).astype(f32)
        bot = (p[y1][:, x0] * (one - wx) + p[y1][:, x1] * wx).astype(f32)
        val = (top * (one - wy) + bot * wy).astype(f32)
        out[c, :, :rw] = (val / f32(127.5) - one).astype(f32)
    return out
