"""Page preprocessing on the B200 (detector resize + normalize, batched ROI
warp) against the reference's own kernels run on the same GPU
(native/src/kernels/detector_preprocess.cu, native/src/kernels/roi_warp.cu,
compiled unmodified into oracle/_ref/) and against the numpy restatement in
oracle/preprocess.py.

Bar: the f32 NCHW output equals the reference kernel's bit for bit; the FP16
NHWC output equals the reference's f32 value rounded to nearest FP16; the
numpy restatement (bit-exact on the committed golden fixtures, its fused
multiply-adds emulated in float64) agrees within 1e-3 absolute on these
larger cases.
"""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import ptr, stream_handle
from helpers import rng
from oracle import preprocess as OP

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_preprocess.so"
P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
F32, F16 = 0, 1
ORACLE_TOL = 1e-3


@pytest.fixture(scope="module")
def ref_pp():
    if not REF.exists():
        pytest.skip("libref_preprocess.so not built (needs the reference sources at build time)")
    lib = ctypes.CDLL(str(REF))
    lib.ref_resize_normalize_detector_padded.argtypes = [P, S, I, I, P, I, I, I, I, I, P]
    lib.ref_batch_roi_warp.argtypes = [P, S, I, I, P, P, P, I, I, I, I, P]
    return lib


def _page(r, h, w, pad=0):
    img = r.integers(0, 256, (h, w, 3), dtype=np.uint8)
    step = w * 3 + pad
    pitched = np.zeros((h, step), np.uint8)
    pitched[:, : w * 3] = img.reshape(h, -1)
    return img, step, torch.from_numpy(pitched).cuda()


DET_CASES = [
    # src h, w, row pad, dst h, w, content h, w, bgr
    (1080, 1920, 0, 960, 960, 540, 960, 0),   # landscape page, aspect kept, padded canvas
    (37, 53, 5, 64, 100, 61, 97, 1),          # upscale, pitched rows, BGR source
    (200, 130, 3, 96, 98, 96, 62, 0),         # canvas width not a multiple of 4
    (31, 29, 0, 32, 32, 32, 32, 1),           # unpadded form
]


@pytest.mark.parametrize("case", DET_CASES)
def test_detector_preprocess_matches_reference(native, cuda, ref_pp, case):
    sh, sw, pad, dh, dw, ch, cw, bgr = case
    img, step, t = _page(rng(300 + sh + dw), sh, sw, pad)
    want = torch.empty(3, dh, dw, dtype=torch.float32, device=cuda)
    got = torch.full_like(want, float("nan"))
    got16 = torch.full((dh, dw, 3), float("nan"), dtype=torch.float16, device=cuda)
    s = stream_handle()
    assert ref_pp.ref_resize_normalize_detector_padded(ptr(t), step, sh, sw, ptr(want), dh, dw, ch, cw, bgr, s) == 0
    if (ch, cw) == (dh, dw):
        rc = native.ppocr_b200_resize_normalize_detector(ptr(t), step, sh, sw, ptr(got), dh, dw, bgr, s)
    else:
        rc = native.ppocr_b200_resize_normalize_detector_padded(ptr(t), step, sh, sw, ptr(got), dh, dw, ch, cw, bgr, s)
    assert rc == 0, native.ppocr_b200_last_error()
    assert native.ppocr_b200_detector_preprocess(ptr(t), step, sh, sw, 0, 1, ptr(got16), dh, dw, ch, cw, bgr, F16,
                                                 s) == 0, native.ppocr_b200_last_error()
    torch.cuda.synchronize()
    assert torch.equal(got, want), f"max diff {(got - want).abs().max().item()}"
    assert torch.equal(got16, want.permute(1, 2, 0).half())
    o = OP.detector_preprocess(img, dh, dw, ch, cw, bool(bgr))
    assert np.abs(o - want.cpu().numpy()).max() <= ORACLE_TOL


def test_detector_preprocess_batch_of_pages(native, cuda, ref_pp):
    r = rng(310)
    pages = [_page(r, 120, 160) for _ in range(3)]
    stack = torch.stack([p[2] for p in pages])  # [3, 120, 480] contiguous pages
    got = torch.empty(3, 64, 96, 3, dtype=torch.float16, device=cuda)
    s = stream_handle()
    assert native.ppocr_b200_detector_preprocess(ptr(stack), 480, 120, 160, 120 * 480, 3, ptr(got), 64, 96, 60,
                                                 80, 0, F16, s) == 0, native.ppocr_b200_last_error()
    for i, (_, step, t) in enumerate(pages):
        want = torch.empty(3, 64, 96, dtype=torch.float32, device=cuda)
        assert ref_pp.ref_resize_normalize_detector_padded(ptr(t), step, 120, 160, ptr(want), 64, 96, 60, 80, 0,
                                                           s) == 0
        torch.cuda.synchronize()
        assert torch.equal(got[i], want.permute(1, 2, 0).half())


def test_detector_preprocess_rejects_bad_arguments(native, cuda):
    t = torch.zeros(10, 30, dtype=torch.uint8, device=cuda)
    y = torch.empty(3, 8, 8, device=cuda)
    s = stream_handle()
    for args in [(ptr(t), 30, 10, 10, ptr(y), 8, 8, 9, 8, 0),    # content taller than the canvas
                 (ptr(t), 29, 10, 10, ptr(y), 8, 8, 8, 8, 0),    # row pitch below cols * 3
                 (None, 30, 10, 10, ptr(y), 8, 8, 8, 8, 0),      # no source
                 (ptr(t), 30, 10, 10, ptr(y), 8, 8, 0, 8, 0)]:   # empty content
        assert native.ppocr_b200_resize_normalize_detector_padded(*args, s) == -1
        assert native.ppocr_b200_last_error() == b"invalid detector preprocess arguments"


def _crops(r, n, page_h, page_w, dst_h, dst_w):
    m, widths = [], []
    for k in range(n):
        wq = r.uniform(40, 400)
        hq = r.uniform(10, 40)
        cx, cy = r.uniform(0, page_w - 40), r.uniform(0, page_h - 20)
        a = np.deg2rad(r.uniform(-30, 30))
        c, s = np.cos(a), np.sin(a)
        quad = np.array([[cx + c * dx - s * dy, cy + s * dx + c * dy]
                         for dx, dy in ((0, 0), (wq, 0), (wq, hq), (0, hq))]) + r.normal(0, 2, (4, 2))
        natural = max(1, int(np.ceil(dst_h * wq / hq)))
        cw = min(dst_w, natural)
        m.append(OP.quad_to_rect_inverse(quad, cw, dst_h))
        widths.append(cw)
    return np.stack(m).astype(np.float32), np.array(widths, np.int32)


@pytest.mark.parametrize("batch,dst_w,bgr", [(64, 320, 0), (17, 318, 1), (5, 64, 0)])
def test_roi_warp_matches_reference(native, cuda, ref_pp, batch, dst_w, bgr):
    r = rng(320 + batch + dst_w)
    img, step, t = _page(r, 960, 960, 0)
    dst_h = 48
    m, widths = _crops(r, batch, 960, 960, dst_h, dst_w)
    if batch == 17:
        # edge cases: out-of-page quads, a degenerate denominator (clamped to
        # 1e-7 -> clamped far coordinates), a non-finite transform, zero
        # crop width, crop width above the canvas
        m[0] = np.array([1, 0, 5000, 0, 1, -3000, 0, 0, 1], np.float32)
        m[1] = np.array([1, 0, 0, 0, 1, 0, 0, 0, 0], np.float32)
        m[2] = np.array([np.inf, 0, 0, 0, 1, 0, 0, 0, 1], np.float32)
        m[3] = np.array([np.nan] * 9, np.float32)
        widths[4] = 0
        widths[5] = dst_w + 50
    tm, tw = torch.from_numpy(m).cuda(), torch.from_numpy(widths).cuda()
    want = torch.empty(batch, 3, dst_h, dst_w, dtype=torch.float32, device=cuda)
    got = torch.full_like(want, float("nan"))
    got16 = torch.full((batch, dst_h, dst_w, 3), float("nan"), dtype=torch.float16, device=cuda)
    s = stream_handle()
    assert ref_pp.ref_batch_roi_warp(ptr(t), step, 960, 960, ptr(tm), ptr(tw), ptr(want), batch, dst_h, dst_w, bgr,
                                     s) == 0
    assert native.ppocr_b200_batch_roi_warp(ptr(t), step, 960, 960, ptr(tm), ptr(tw), ptr(got), batch, dst_h, dst_w,
                                            bgr, s) == 0, native.ppocr_b200_last_error()
    assert native.ppocr_b200_roi_warp(ptr(t), step, 960, 960, ptr(tm), ptr(tw), ptr(got16), batch, dst_h, dst_w,
                                      bgr, F16, s) == 0, native.ppocr_b200_last_error()
    torch.cuda.synchronize()
    assert torch.equal(got, want), f"max diff {(got - want).abs().max().item()}"
    assert torch.equal(got16, want.permute(0, 2, 3, 1).half())
    o = OP.roi_warp(img, m, widths, dst_h, dst_w, bool(bgr))
    assert np.abs(o - want.cpu().numpy()).max() <= ORACLE_TOL


def test_roi_warp_empty_batch_is_noop(native, cuda):
    assert native.ppocr_b200_batch_roi_warp(None, 0, 0, 0, None, None, None, 0, 48, 320, 0, stream_handle()) == 0
