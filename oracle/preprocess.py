"""numpy float32 restatement of the page preprocessing (test oracle only).

detector_preprocess  native/src/kernels/detector_preprocess.cu:12-73
roi_warp             native/src/kernels/roi_warp.cu:10-109

Every operation is a float32 operation in the reference's order. Where the
reference writes `a * b + c`, its compiler fuses the multiply and the add
into one rounding (an FMA; in `a*b + c*d` the left product is the fused one,
in a chain of sums each further product is fused into the running sum), and
`fma()` below restates that: the product is exact in float64 and the sum is
rounded once more to float32 (a double rounding that differs from a true
FMA only in rare ties). The pad colour of the detector canvas is a constant
expression, evaluated without fusion. With these the restatement matches the
reference kernels' output bit for bit on the golden fixtures.
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


def fma(a, b, c):
    """float32 fused multiply-add: round32(a * b + c)."""
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(f32)


def mul(a, b):
    return (np.asarray(a, f32) * np.asarray(b, f32)).astype(f32)

MEAN_BGR = (f32(0.485), f32(0.456), f32(0.406))
STD_BGR = (f32(0.229), f32(0.224), f32(0.225))


def _bilinear(img, xs, ys, ch):
    """detector_preprocess.cu:12-33 for one channel at float32 coords."""
    h, w = img.shape[:2]
    x0u = np.floor(xs).astype(np.int64)
    y0u = np.floor(ys).astype(np.int64)
    wx = (xs - x0u.astype(f32)).astype(f32)
    wy = (ys - y0u.astype(f32)).astype(f32)
    x0 = np.clip(x0u, 0, w - 1)
    x1 = np.clip(x0u + 1, 0, w - 1)
    y0 = np.clip(y0u, 0, h - 1)
    y1 = np.clip(y0u + 1, 0, h - 1)
    c = img[..., ch].astype(f32)
    one = f32(1.0)
    top = fma(c[y0, x0], one - wx, mul(c[y0, x1], wx))
    bot = fma(c[y1, x0], one - wx, mul(c[y1, x1], wx))
    return fma(top, one - wy, mul(bot, wy))


def detector_preprocess(img: np.ndarray, dst_h: int, dst_w: int, content_h: int, content_w: int,
                        source_is_bgr: bool) -> np.ndarray:
    """u8 [H, W, 3] page -> f32 [3, dst_h, dst_w] (channel order B, G, R)."""
    h, w = img.shape[:2]
    sx_scale = f32(w) / f32(content_w)
    sy_scale = f32(h) / f32(content_h)
    ys, xs = np.meshgrid(np.arange(dst_h, dtype=f32), np.arange(dst_w, dtype=f32), indexing="ij")
    src_x = fma(xs + f32(0.5), sx_scale, f32(-0.5))
    src_y = fma(ys + f32(0.5), sy_scale, f32(-0.5))
    pad = (xs >= content_w) | (ys >= content_h)
    chans = (0, 1, 2) if source_is_bgr else (2, 1, 0)
    out = np.empty((3, dst_h, dst_w), f32)
    inv255 = f32(1.0) / f32(255.0)
    for k, ch in enumerate(chans):
        inside = (fma(_bilinear(img, src_x, src_y, ch), inv255, -MEAN_BGR[k]) / STD_BGR[k]).astype(f32)
        white = ((f32(255.0) * inv255 - MEAN_BGR[k]) / STD_BGR[k]).astype(f32)
        out[k] = np.where(pad, white, inside)
    return out


def roi_warp(img: np.ndarray, m_invs: np.ndarray, crop_widths: np.ndarray, dst_h: int, dst_w: int,
             output_bgr: bool) -> np.ndarray:
    """u8 [H, W, 3] page, m_invs [B, 9], crop_widths [B] -> f32 [B, 3, dst_h, dst_w]."""
    h, w = img.shape[:2]
    B = m_invs.shape[0]
    out = np.zeros((B, 3, dst_h, dst_w), f32)
    ys, xs = np.meshgrid(np.arange(dst_h, dtype=f32), np.arange(dst_w, dtype=f32), indexing="ij")
    one = f32(1.0)
    planes = [img[..., c].astype(f32) for c in range(3)]
    for b in range(B):
        m = m_invs[b].astype(f32)
        den = (fma(m[6], xs, mul(m[7], ys)) + m[8]).astype(f32)
        small = np.abs(den) < f32(1e-7)
        den = np.where(small, np.where(den < 0, f32(-1e-7), f32(1e-7)), den).astype(f32)
        with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
            inv = (one / den).astype(f32)
            sx = ((fma(m[0], xs, mul(m[1], ys)) + m[2]).astype(f32) * inv).astype(f32)
            sy = ((fma(m[3], xs, mul(m[4], ys)) + m[5]).astype(f32) * inv).astype(f32)
        keep = (xs < crop_widths[b]) & np.isfinite(sx) & np.isfinite(sy)
        sx = np.clip(np.where(keep, sx, 0), f32(-1.0), f32(w + 1)).astype(f32)
        sy = np.clip(np.where(keep, sy, 0), f32(-1.0), f32(h + 1)).astype(f32)
        xi = np.floor(sx).astype(np.int64)
        yi = np.floor(sy).astype(np.int64)
        ax = (sx - xi.astype(f32)).astype(f32)
        ay = (sy - yi.astype(f32)).astype(f32)
        x0, x1 = np.clip(xi, 0, w - 1), np.clip(xi + 1, 0, w - 1)
        y0, y1 = np.clip(yi, 0, h - 1), np.clip(yi + 1, 0, h - 1)
        w00 = ((one - ax) * (one - ay)).astype(f32)
        w10 = (ax * (one - ay)).astype(f32)
        w01 = ((one - ax) * ay).astype(f32)
        w11 = (ax * ay).astype(f32)
        vals = []
        for c in range(3):
            p = planes[c]
            acc = fma(w00, p[y0, x0], mul(w10, p[y0, x1]))
            acc = fma(w01, p[y1, x0], acc)
            vals.append(fma(w11, p[y1, x1], acc))
        order = (2, 1, 0) if output_bgr else (0, 1, 2)
        inv127 = f32(1.0) / f32(127.5)
        for k, c in enumerate(order):
            out[b, k] = np.where(keep, fma(vals[c], inv127, -one), f32(0.0))
    return out


def quad_to_rect_inverse(quad: np.ndarray, crop_w: int, crop_h: int) -> np.ndarray:
    """Row-major 3x3 homography mapping crop pixel (x, y) to page coordinates
    for the quadrilateral quad [4, 2] (top-left, top-right, bottom-right,
    bottom-left) onto a crop_w x crop_h rectangle -- the m_inv a caller passes
    per crop (the reference's host computes it in compute_crop_transform,
    native/include/ppocrv6_native/common/perspective.h:50-83, from the same
    four correspondences). Solved here in float64; used to make test inputs."""
    dst = np.array([[0, 0], [crop_w - 1, 0], [crop_w - 1, crop_h - 1], [0, crop_h - 1]], np.float64)
    src = np.asarray(quad, np.float64)
    A, rhs = [], []
    for (x, y), (u, v) in zip(dst, src):
        A.append([x, y, 1, 0, 0, 0, -u * x, -u * y])
        rhs.append(u)
        A.append([0, 0, 0, x, y, 1, -v * x, -v * y])
        rhs.append(v)
    h = np.linalg.solve(np.array(A), np.array(rhs))
    return np.append(h, 1.0).astype(np.float32)
