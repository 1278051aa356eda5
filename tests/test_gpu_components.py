"""DB post-processing front end on the B200 (8-connected components of the
binarized map with per-component box statistics) against the oracle in
oracle/components.py, which is pinned to OpenCV's own
connectedComponentsWithStats output by tests/test_cpu_golden.py.

Bar: labels, counts, (left, top, width, height, area) and the 32.32
fixed-point probability sums bit-exact."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import ptr, stream_handle
from helpers import rng
from oracle import components as OC

pytestmark = pytest.mark.gpu


def run(native, cuda, bitmaps, probs, max_comp, with_prob=True):
    pages, h, w = bitmaps.shape
    bm = torch.from_numpy(bitmaps).cuda()
    pr = torch.from_numpy(probs).cuda()
    labels = torch.full((pages, h, w), -7, dtype=torch.int32, device=cuda)
    counts = torch.full((pages,), -7, dtype=torch.int32, device=cuda)
    stats = torch.full((pages, max_comp, 5), -7, dtype=torch.int32, device=cuda)
    q = torch.zeros((pages, max_comp), dtype=torch.int64, device=cuda)
    wsb = native.ppocr_b200_db_components_workspace(pages, h, w, max_comp)
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda)
    rc = native.ppocr_b200_db_components(ptr(bm), ptr(pr) if with_prob else None, pages, h, w, max_comp,
                                         ptr(labels), ptr(counts), ptr(stats), ptr(q), ptr(ws), stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    torch.cuda.synchronize()
    return labels.cpu().numpy(), counts.cpu().numpy(), stats.cpu().numpy(), q.cpu().numpy().view(np.uint64)


def check(native, cuda, bitmaps, probs, max_comp=4096, with_prob=True):
    labels, counts, stats, q = run(native, cuda, bitmaps, probs, max_comp, with_prob)
    for p in range(bitmaps.shape[0]):
        wl, wn, ws, wq = OC.components(bitmaps[p], probs[p] if with_prob else None)
        assert counts[p] == wn, f"page {p}: {counts[p]} components, oracle {wn}"
        assert np.array_equal(labels[p], wl), f"page {p}: labels differ"
        k = min(wn, max_comp)
        assert np.array_equal(stats[p, :k], ws[:k]), f"page {p}: stats differ"
        assert np.all(stats[p, k:] == 0)
        assert np.array_equal(q[p, :k], wq[:k]), f"page {p}: probability sums differ"
    return counts


def test_components_full_size_pages(native, cuda):
    """BASELINE config 5's 8 pages of 960^2, DB-like maps binarized at 0.3."""
    from ppocr_b200 import workloads

    probs = workloads.db_like_maps(rng(700), 8, 960)
    bitmaps = (probs > np.float32(0.3)).astype(np.uint8) * 255
    counts = check(native, cuda, bitmaps, probs)
    assert counts.min() > 10


@pytest.mark.parametrize("pages,h,w", [(3, 37, 53), (2, 1, 1), (1, 1, 1000), (2, 513, 2)])
def test_components_odd_shapes(native, cuda, pages, h, w):
    """Odd heights and widths (padding keys of the 2x2 blocks), single rows,
    single columns, pages whose keys straddle scan blocks."""
    r = rng(710 + h + w)
    probs = r.uniform(0, 0.6, (pages, h, w)).astype(np.float32)
    bitmaps = (probs > np.float32(0.3)).astype(np.uint8)
    check(native, cuda, bitmaps, probs)


def test_components_edge_patterns(native, cuda):
    h, w = 24, 31
    pages = []
    pages.append(np.zeros((h, w), np.uint8))                                  # nothing
    pages.append(np.ones((h, w), np.uint8))                                   # one component, the page
    pages.append((np.indices((h, w)).sum(0) % 2).astype(np.uint8))            # diagonal-only connectivity
    corners = np.zeros((h, w), np.uint8)
    corners[0, 0] = corners[0, -1] = corners[-1, 0] = corners[-1, -1] = 1      # single pixels at corners
    pages.append(corners)
    spiral = np.zeros((h, w), np.uint8)                                       # one long, winding component
    spiral[1, 1:-1] = spiral[1:-1, -2] = spiral[-2, 2:-1] = spiral[3:-1, 2] = spiral[3, 2:-3] = 1
    pages.append(spiral)
    bitmaps = np.stack(pages)
    probs = rng(720).uniform(0, 1, bitmaps.shape).astype(np.float32)
    counts = check(native, cuda, bitmaps, probs)
    assert counts.tolist() == [0, 1, 1, 4, 1]


def test_components_overflow_and_no_prob(native, cuda):
    """More components than max_components: all are labelled and counted,
    only the first max_components get statistics; prob may be null."""
    r = rng(730)
    bitmaps = (r.uniform(0, 1, (2, 64, 64)) > 0.8).astype(np.uint8)
    probs = np.zeros(bitmaps.shape, np.float32)
    counts = check(native, cuda, bitmaps, probs, max_comp=5, with_prob=False)
    assert counts.min() > 5


def test_components_rejects_bad_arguments(native, cuda):
    assert native.ppocr_b200_db_components(None, None, 1, 4, 4, 8, None, None, None, None, None,
                                           stream_handle()) == -1
    assert b"invalid" in native.ppocr_b200_last_error()
