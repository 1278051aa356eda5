"""Makes the golden fixtures in this folder from the reference's OWN code.

The reference sources are compiled unmodified into oracle/_ref/ by
oracle/Makefile (`make -C oracle ref`, where the reference tree is present);
this script runs them on small seeded inputs and stores inputs + outputs as
compressed .npz files, so the CPU tests can pin the oracle against real
reference outputs without a GPU or the reference tree.

  python tests/golden/make_golden.py cpu            # ctc_collapse.npz (host code),
                                                    # components.npz (OpenCV)
  python tests/golden/make_golden.py gpu [--out D]  # classifier / depthwise /
                                                    # pool / preprocess .npz
                                                    # (reference CUDA kernels,
                                                    # needs a B200)

Sources of each fixture:
  ctc_collapse.npz  native/src/recognition/ctc_decode.cpp:7-81
  classifier.npz    native/src/kernels/classifier.cu:611-680 (WMMA path)
  depthwise.npz     native/src/compiled/spatial_kernels.cuh depthwise_nhwc_vec8
  pool.npz          native/src/compiled/spatial_kernels.cuh pool_nhwc_vec8
  preprocess.npz    native/src/kernels/detector_preprocess.cu:84-101,
                    native/src/kernels/roi_warp.cu:113-131
  components.npz    OpenCV connectedComponentsWithStats (connectivity 8) on
                    binarized DB-like maps: the library the reference's
                    db_postprocess.cpp:183-252 runs on these maps
"""

from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = REPO / "oracle" / "_ref"
SEED = 20261201
P, I = ctypes.c_void_p, ctypes.c_int


def _lib(name):
    path = REF / name
    if not path.exists():
        sys.exit(f"{path} missing: build it with `make -C oracle ref` where the reference tree is present")
    return ctypes.CDLL(str(path))


def make_cpu(out: Path) -> None:
    lib = _lib("libref_ctc.so")
    lib.ref_ctc_decode_batch.argtypes = [P, P, I, I, I, P, P, P]
    r = np.random.default_rng(SEED + 900)
    lines, T = 96, 40
    ids = r.integers(0, 6, (lines, T)).astype(np.int32)
    ids[::5] = 0                                     # all-blank lines
    ids[1::7] = r.integers(0, 18385, (len(ids[1::7]), T))
    ids[2::9, :] = ids[2::9, :1]                     # one long repeat
    ids[3, :4] = [7, 0, 7, 7]                        # repeat split by a blank
    ids[4, :2] = [-3, 99999]                         # out-of-vocabulary ids
    scores = r.random((lines, T)).astype(np.float32)
    o_ids = np.empty((lines, T), np.int32)
    o_len = np.empty(lines, np.int32)
    o_sc = np.empty(lines, np.float32)
    assert lib.ref_ctc_decode_batch(ids.ctypes.data, scores.ctypes.data, lines, T, 0, o_ids.ctypes.data,
                                    o_len.ctypes.data, o_sc.ctypes.data) == 0
    np.savez_compressed(out / "ctc_collapse.npz", ids=ids, scores=scores, blank=np.int32(0),
                        out_ids=o_ids, out_len=o_len, out_score=o_sc)
    make_components(out)


def db_like_map(r, h, w, blobs=40):
    """float32 [h, w] in [0, 1]: rotated elongated text-line blobs plus
    speckle, the shapes a DB probability map has."""
    yy, xx = np.mgrid[0:h, 0:w].astype(np.float32)
    m = np.zeros((h, w), np.float32)
    for _ in range(blobs):
        cy, cx = r.uniform(0, h), r.uniform(0, w)
        a = r.uniform(-0.4, 0.4)
        lw, lh = r.uniform(4, w / 3), r.uniform(1.5, 6)
        u = (xx - cx) * np.cos(a) + (yy - cy) * np.sin(a)
        v = -(xx - cx) * np.sin(a) + (yy - cy) * np.cos(a)
        m = np.maximum(m, np.exp(-((u / lw) ** 8 + (v / lh) ** 2)))
    m += r.uniform(0, 0.35, (h, w)).astype(np.float32)  # speckle around the 0.3 threshold
    return np.clip(m, 0, 1).astype(np.float32)


def make_components(out: Path) -> None:
    import cv2

    r = np.random.default_rng(SEED + 902)
    res = {}
    cases = {"dblike_96x128": db_like_map(r, 96, 128), "dblike_37x53": db_like_map(r, 37, 53, 8)}
    checker = np.indices((9, 11)).sum(0) % 2  # diagonal-only connectivity
    cases["checker_9x11"] = checker.astype(np.float32)
    for name, prob in cases.items():
        bitmap = (prob > np.float32(0.3)).astype(np.uint8) * 255
        n, labels, stats, _ = cv2.connectedComponentsWithStats(bitmap, connectivity=8, ltype=cv2.CV_32S)
        res[f"{name}__prob"] = prob
        res[f"{name}__bitmap"] = bitmap
        res[f"{name}__labels"] = labels.astype(np.int32)
        res[f"{name}__stats"] = stats[1:].astype(np.int32)  # row 0 is the background
    np.savez_compressed(out / "components.npz", **res)


def make_gpu(out: Path) -> None:
    import torch

    dev = torch.device("cuda:0")
    s = P(torch.cuda.current_stream().cuda_stream)
    ptr = lambda t: P(t.data_ptr())  # noqa: E731
    r = np.random.default_rng(SEED + 901)

    # ---- classifier (reference WMMA path: H % 16 == 0, V a multiple of 16)
    cls = _lib("libref_classifier.so")
    cls.ref_classifier_workspace.argtypes = [I, I, I, I, ctypes.POINTER(ctypes.c_size_t)]
    cls.ref_linear_argmax_prob_wmma.argtypes = [P, P, P, P, P, P, I, I, I, I, P, P, P, I, P]
    rows, H, V = 80, 128, 1008
    hid = r.standard_normal((rows, H)).astype(np.float16)
    w = (r.uniform(-1, 1, (H, V)) * np.sqrt(6.0 / (H + V)) * 4).astype(np.float16)
    b = r.normal(0, 0.1, V).astype(np.float16)
    dh, dw, db = (torch.from_numpy(a).to(dev) for a in (hid, w, b))
    cnt = ctypes.c_size_t()
    assert cls.ref_classifier_workspace(rows, V, 16, 512, ctypes.byref(cnt)) == 0
    part = [torch.empty(cnt.value, dtype=t, device=dev) for t in (torch.int32, torch.float32, torch.float32)]
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    prob = torch.empty(rows, dtype=torch.float32, device=dev)
    mx = torch.empty(rows, dtype=torch.float32, device=dev)
    assert cls.ref_linear_argmax_prob_wmma(ptr(dh), ptr(dw), ptr(db), ptr(ids), ptr(prob), ptr(mx), rows, H, V,
                                           512, ptr(part[0]), ptr(part[1]), ptr(part[2]), 1, s) == 0
    torch.cuda.synchronize()
    np.savez_compressed(out / "classifier.npz", hidden=hid, weight=w, bias=b, ids=ids.cpu().numpy(),
                        prob=prob.cpu().numpy(), max_logit=mx.cpu().numpy())

    # ---- depthwise + pools (reference NHWC kernels)
    sp = _lib("libref_spatial.so")
    sp.ref_depthwise_nhwc.argtypes = [P, P, P, P] + [I] * 13 + [P]
    sp.ref_pool_nhwc.argtypes = [P, P, I, I, I, I, I, I, I, P]
    dw_cases = {}
    for name, (B, C, Hh, W, kh, kw, sh, sw, act) in {
        "dw5x5_s1_none": (1, 16, 9, 13, 5, 5, 1, 1, 0),
        "dw3x3_s2_relu": (2, 8, 11, 10, 3, 3, 2, 2, 1),
        "dw3x3_s21_gelu": (1, 24, 7, 9, 3, 3, 2, 1, 2),
        "dw1x7_s1_relu": (1, 8, 5, 17, 1, 7, 1, 1, 1),
    }.items():
        ph, pw = kh // 2, kw // 2
        OH, OW = (Hh + 2 * ph - kh) // sh + 1, (W + 2 * pw - kw) // sw + 1
        x = r.uniform(-2, 2, (B, Hh, W, C)).astype(np.float16)
        wt = r.normal(0, 0.4, (C, kh, kw)).astype(np.float16)
        bias = r.normal(0, 0.2, C).astype(np.float16)
        tx, tw, tb = (torch.from_numpy(a).to(dev) for a in (x, wt, bias))
        y = torch.empty(B, OH, OW, C, dtype=torch.float16, device=dev)
        assert sp.ref_depthwise_nhwc(ptr(tx), ptr(tw), ptr(tb), ptr(y), B, C, Hh, W, OH, OW, kh, kw, sh, sw, ph, pw,
                                     act, s) == 0
        torch.cuda.synchronize()
        dw_cases[name] = (x, wt, bias, np.array([kh, kw, sh, sw, ph, pw, act], np.int32), y.cpu().numpy())
    np.savez_compressed(out / "depthwise.npz", **{f"{k}__{f}": v for k, vals in dw_cases.items()
                                                  for f, v in zip(("x", "w", "bias", "geom", "y"), vals)})
    pools = {}
    for kind, (B, C, Hh, W) in ((0, (1, 16, 6, 9)), (1, (2, 32, 3, 10))):
        k, st = ((2, 2), (1, 1)) if kind == 0 else ((3, 2), (3, 2))
        OH, OW = (Hh - k[0]) // st[0] + 1, (W - k[1]) // st[1] + 1
        x = r.uniform(-3, 3, (B, Hh, W, C)).astype(np.float16)
        tx = torch.from_numpy(x).to(dev)
        y = torch.empty(B, OH, OW, C, dtype=torch.float16, device=dev)
        assert sp.ref_pool_nhwc(ptr(tx), ptr(y), B, C, Hh, W, OH, OW, kind, s) == 0
        torch.cuda.synchronize()
        pools[f"kind{kind}__x"] = x
        pools[f"kind{kind}__y"] = y.cpu().numpy()
    np.savez_compressed(out / "pool.npz", **pools)

    # ---- page preprocessing (reference detector resize/normalize + ROI warp)
    pp = _lib("libref_preprocess.so")
    pp.ref_resize_normalize_detector_padded.argtypes = [P, ctypes.c_size_t, I, I, P, I, I, I, I, I, P]
    pp.ref_batch_roi_warp.argtypes = [P, ctypes.c_size_t, I, I, P, P, P, I, I, I, I, P]
    page = r.integers(0, 256, (37, 53, 3), dtype=np.uint8)
    step = 53 * 3 + 5  # padded row pitch
    pitched = np.zeros((37, step), np.uint8)
    pitched[:, : 53 * 3] = page.reshape(37, -1)
    tp = torch.from_numpy(pitched).to(dev)
    det = {}
    for name, (dh_, dw_, ch, cw, bgr) in {"up_padded_rgb": (64, 100, 61, 97, 0),
                                          "down_bgr": (24, 36, 24, 36, 1)}.items():
        y = torch.empty(3, dh_, dw_, dtype=torch.float32, device=dev)
        assert pp.ref_resize_normalize_detector_padded(ptr(tp), step, 37, 53, ptr(y), dh_, dw_, ch, cw, bgr, s) == 0
        torch.cuda.synchronize()
        det[f"det_{name}__geom"] = np.array([dh_, dw_, ch, cw, bgr], np.int32)
        det[f"det_{name}__y"] = y.cpu().numpy()
    src = r.integers(0, 256, (96, 128, 3), dtype=np.uint8)
    ts = torch.from_numpy(src).to(dev)
    m_invs, widths = [], []
    for k in range(6):
        cx, cy = 20 + 15 * k, 30 + 8 * k
        ang = np.deg2rad(-20 + 8 * k)
        wq, hq = 50 + 5 * k, 12 + k
        c, si = np.cos(ang), np.sin(ang)
        quad = np.array([[cx + c * dx - si * dy, cy + si * dx + c * dy]
                         for dx, dy in ((0, 0), (wq, 0), (wq, hq), (0, hq))])
        quad += r.normal(0, 1.5, quad.shape)
        m = _homography(quad, 60, 16)
        m_invs.append(m)
        widths.append(min(64, 40 + 6 * k))
    m_invs[5] = np.array([1, 0, 0, 0, 1, 0, 0, 0, 0], np.float32)  # degenerate denominator
    mi = np.stack(m_invs).astype(np.float32)
    cw_ = np.array(widths, np.int32)
    tm, tw = torch.from_numpy(mi).to(dev), torch.from_numpy(cw_).to(dev)
    for bgr in (0, 1):
        y = torch.empty(6, 3, 16, 64, dtype=torch.float32, device=dev)
        assert pp.ref_batch_roi_warp(ptr(ts), 128 * 3, 96, 128, ptr(tm), ptr(tw), ptr(y), 6, 16, 64, bgr, s) == 0
        torch.cuda.synchronize()
        det[f"roi_bgr{bgr}__y"] = y.cpu().numpy()
    np.savez_compressed(out / "preprocess.npz", page=page, roi_src=src, m_invs=mi, crop_widths=cw_, **det)


def _homography(quad, crop_w, crop_h):
    dst = np.array([[0, 0], [crop_w - 1, 0], [crop_w - 1, crop_h - 1], [0, crop_h - 1]], np.float64)
    A, rhs = [], []
    for (x, y), (u, v) in zip(dst, np.asarray(quad, np.float64)):
        A += [[x, y, 1, 0, 0, 0, -u * x, -u * y], [0, 0, 0, x, y, 1, -v * x, -v * y]]
        rhs += [u, v]
    return np.append(np.linalg.solve(np.array(A), np.array(rhs)), 1.0).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["cpu", "gpu"])
    ap.add_argument("--out", default=str(HERE))
    a = ap.parse_args()
    out = Path(a.out)
    out.mkdir(parents=True, exist_ok=True)
    (make_cpu if a.what == "cpu" else make_gpu)(out)
    print("wrote", sorted(p.name for p in out.glob("*.npz")))


if __name__ == "__main__":
    main()
