"""Seeded synthetic inputs of the five benchmark configurations.

No public dataset is involved: each generator draws the shapes and value
distributions the configuration names (NumPy PCG64, seed given by the
caller). C1 is the CTC head on materialised logits, C2 the depthwise-
separable NHWC block, C3 the SVTR neck, C4 the full recognizer, C5 the page
pipeline (detector + binarize + recognizer on 64 line crops per page).
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
