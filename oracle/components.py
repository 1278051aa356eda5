"""CPU restatement of the DB post-processing front end (test oracle only).

8-connected components of a binarized map with (left, top, width, height,
area) per component, numbered the way OpenCV's
connectedComponentsWithStats(connectivity=8) numbers them (OpenCV is the
library the reference's db_postprocess.cpp:183-252 runs on these maps): in
order of each component's first pixel in 2x2-block raster order (blocks of
rows 2b, 2b+1 scanned left to right, then the pixel's place in its block),
which is how OpenCV's block-based labelling hands out provisional labels.
The golden fixture tests/golden/components.npz holds OpenCV's own output
for the CPU tests. scipy.ndimage.label finds the components here; the
probability sums are the device's 32.32 fixed point: sum of
floor(clamp(p, 0, 1) * 2^32) over each component's pixels.
"""

from __future__ import annotations

import numpy as np
from scipy import ndimage


def components(bitmap: np.ndarray, prob: np.ndarray | None = None):
    """bitmap [h, w] (non-zero = foreground) -> (labels int32 [h, w], count,
    stats int32 [count, 5], prob_sum_q32 uint64 [count])."""
    fg = bitmap != 0
    raw, count = ndimage.label(fg, structure=np.ones((3, 3), np.int32))
    labels = np.zeros(raw.shape, np.int32)
    if count:
        ys, xs = np.nonzero(fg)
        wb = (fg.shape[1] + 1) // 2
        key = ((ys >> 1) * wb + (xs >> 1)) * 4 + (ys & 1) * 2 + (xs & 1)
        first = np.full(count + 1, np.iinfo(np.int64).max)
        np.minimum.at(first, raw[ys, xs], key)
        remap = np.zeros(count + 1, np.int32)
        remap[np.argsort(first[1:], kind="stable") + 1] = np.arange(1, count + 1, dtype=np.int32)
        labels = remap[raw]
    stats = np.zeros((count, 5), np.int32)
    q = np.zeros(count, np.uint64)
    if count:
        ys, xs = np.nonzero(fg)
        ids = labels[ys, xs] - 1
        stats[:, 0] = np.full(count, np.iinfo(np.int32).max)
        stats[:, 1] = np.full(count, np.iinfo(np.int32).max)
        np.minimum.at(stats[:, 0], ids, xs)
        np.minimum.at(stats[:, 1], ids, ys)
        x1 = np.full(count, -1, np.int64)
        y1 = np.full(count, -1, np.int64)
        np.maximum.at(x1, ids, xs)
        np.maximum.at(y1, ids, ys)
        stats[:, 2] = x1 - stats[:, 0] + 1
        stats[:, 3] = y1 - stats[:, 1] + 1
        stats[:, 4] = np.bincount(ids, minlength=count)
        if prob is not None:
            p = np.clip(prob[ys, xs].astype(np.float64), 0.0, 1.0)
            fixed = np.floor(p * 4294967296.0).astype(np.uint64)
            np.add.at(q, ids, fixed)
    return labels, count, stats, q
