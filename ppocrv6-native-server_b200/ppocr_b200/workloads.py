"""Seeded synthetic inputs of the five benchmark configurations.

No public dataset is involved: each generator draws the shapes and value
distributions the configuration names (NumPy PCG64, seed given by the
caller). C1 is the CTC head on materialised logits, C2 the depthwise-
separable NHWC block, C3 the SVTR neck, C4 the full recognizer, C5 the page
pipeline (detector + binarize + recognizer on 64 line crops per page). The
preprocessing workload (decoded u8 pages and per-crop inverse homographies)
feeds the device detector resize/normalize and the batched ROI warp.
"""

from __future__ import annotations

import numpy as np

SEED = 20261201
LINE_H, LINE_W = 48, 320
SEQ, VOCAB = 40, 18385
PAGE = 960
LINES_PER_PAGE = 64


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def c1_logits(r: np.random.Generator, lines: int = 32, T: int = SEQ, V: int = VOCAB) -> np.ndarray:
    """FP16 logits [lines, T, V] ~ N(0,1); one seeded class per timestep
    boosted by +4, 30% of timesteps forced to blank (0), 20% repeating the
    previous timestep's class (so the collapse has repeats to merge)."""
    logits = r.standard_normal((lines, T, V)).astype(np.float32)
    cls = r.integers(1, V, (lines, T))
    blank = r.random((lines, T)) < 0.3
    rep = r.random((lines, T)) < 0.2
    for t in range(1, T):
        cls[:, t] = np.where(rep[:, t], cls[:, t - 1], cls[:, t])
    cls = np.where(blank, 0, cls)
    boosted = np.take_along_axis(logits, cls[..., None], -1) + 4.0
    np.put_along_axis(logits, cls[..., None], boosted, -1)
    return logits.astype(np.float16)


def uniform_nhwc(r: np.random.Generator, shape) -> np.ndarray:
    """FP16 NHWC tensor ~ U(-1, 1) (C2 block input, C4 lines, C5 pages)."""
    return r.uniform(-1.0, 1.0, shape).astype(np.float16)


def c2_input(r: np.random.Generator, batch: int = 16) -> np.ndarray:
    return uniform_nhwc(r, (batch, LINE_H, LINE_W, 64))


def c3_tokens(r: np.random.Generator, lines: int = 256) -> np.ndarray:
    """FP16 neck tokens [lines, 40, 120] ~ N(0,1)."""
    return r.standard_normal((lines, SEQ, 120)).astype(np.float16)


def c4_lines(r: np.random.Generator, lines: int) -> np.ndarray:
    return uniform_nhwc(r, (lines, LINE_H, LINE_W, 3))


def c5_pages(r: np.random.Generator, pages: int = 8, size: int = PAGE):
    """(pages FP16 NHWC [pages, size, size, 3], line crops FP16 NHWC
    [pages * 64, 48, 320, 3]); both ~ U(-1, 1)."""
    return (uniform_nhwc(r, (pages, size, size, 3)),
            uniform_nhwc(r, (pages * LINES_PER_PAGE, LINE_H, LINE_W, 3)))


SOURCE_H, SOURCE_W = 1080, 1920  # decoded page size of the preprocessing workload


def source_pages(r: np.random.Generator, pages: int = 8, h: int = SOURCE_H, w: int = SOURCE_W) -> np.ndarray:
    """Decoded u8 RGB pages [pages, h, w, 3], uniform bytes."""
    return r.integers(0, 256, (pages, h, w, 3), dtype=np.uint8)


def _inverse_homography(quad: np.ndarray, crop_w: int, crop_h: int) -> np.ndarray:
    """Row-major 3x3 map from crop pixel (x, y) to page coordinates for the
    quadrilateral `quad` (4 corners clockwise from top-left), solved from the
    four corner correspondences (the quantity the reference's host computes
    in compute_crop_transform, native/include/ppocrv6_native/common/
    perspective.h:50-83)."""
    dst = np.array([[0, 0], [crop_w - 1, 0], [crop_w - 1, crop_h - 1], [0, crop_h - 1]], np.float64)
    A, rhs = [], []
    for (x, y), (u, v) in zip(dst, np.asarray(quad, np.float64)):
        A += [[x, y, 1, 0, 0, 0, -u * x, -u * y], [0, 0, 0, x, y, 1, -v * x, -v * y]]
        rhs += [u, v]
    return np.append(np.linalg.solve(np.array(A), np.array(rhs)), 1.0).astype(np.float32)


def line_boxes(r: np.random.Generator, n: int, page_h: int, page_w: int, crop_h: int = LINE_H,
               bucket_w: int = LINE_W):
    """n synthetic text-line quadrilaterals on a page (widths 60-600 px,
    heights 16-48 px, rotated up to +-15 degrees, corners jittered), returned
    as (m_invs float32 [n, 9], crop_widths int32 [n]) for a crop_h x bucket_w
    crop: crop width = min(bucket, ceil(crop_h * width / height))."""
    m, widths = [], []
    for _ in range(n):
        wq, hq = r.uniform(60, 600), r.uniform(16, 48)
        cx, cy = r.uniform(0, page_w - wq), r.uniform(0, page_h - hq)
        a = np.deg2rad(r.uniform(-15, 15))
        c, s = np.cos(a), np.sin(a)
        quad = np.array([[cx + c * dx - s * dy, cy + s * dx + c * dy]
                         for dx, dy in ((0, 0), (wq, 0), (wq, hq), (0, hq))]) + r.normal(0, 1.5, (4, 2))
        cw = min(bucket_w, max(1, int(np.ceil(crop_h * wq / hq))))
        m.append(_inverse_homography(quad, cw, crop_h))
        widths.append(cw)
    return np.stack(m), np.array(widths, np.int32)


def db_like_maps(r: np.random.Generator, pages: int = 8, size: int = PAGE, lines: int = LINES_PER_PAGE) -> np.ndarray:
    """Synthetic DB probability maps float32 [pages, size, size] in [0, 1]:
    `lines` rotated text-line blobs per page (soft-edged, 8-40 px tall, up to
    a sixth of the page wide) over a background below the 0.3 threshold with
    0.05 % isolated speckle pixels above it (~460 one-pixel components per
    page), the shapes the binarize + component front end sees."""
    out = np.empty((pages, size, size), np.float32)
    for p in range(pages):
        m = r.uniform(0.0, 0.25, (size, size)).astype(np.float32)
        speck = r.random((size, size)) < 5e-4
        m[speck] = r.uniform(0.3, 0.5, int(speck.sum())).astype(np.float32)
        for _ in range(lines):
            cy, cx = r.uniform(0, size), r.uniform(0, size)
            a = r.uniform(-0.3, 0.3)
            lw, lh = r.uniform(10, size / 6), r.uniform(4, 20)
            ext = int(lw + lh) + 2
            y0, y1 = max(0, int(cy) - ext), min(size, int(cy) + ext)
            x0, x1 = max(0, int(cx) - ext), min(size, int(cx) + ext)
            yy, xx = np.mgrid[y0:y1, x0:x1].astype(np.float32)
            u = (xx - cx) * np.cos(a) + (yy - cy) * np.sin(a)
            v = -(xx - cx) * np.sin(a) + (yy - cy) * np.cos(a)
            blob = np.exp(-((u / lw) ** 8 + (v / lh) ** 2)).astype(np.float32)
            m[y0:y1, x0:x1] = np.maximum(m[y0:y1, x0:x1], blob)
        out[p] = m
    return out
