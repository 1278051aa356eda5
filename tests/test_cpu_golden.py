"""CPU tests: the oracle against golden fixtures made by running the
reference's OWN code (tests/golden/make_golden.py: ctc_decode.cpp on the
host; classifier.cu, spatial_kernels.cuh, detector_preprocess.cu and
roi_warp.cu on a B200). No GPU and no reference tree needed here."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import components as OC
from oracle import layers as L
from oracle import preprocess as OP

GOLDEN = Path(__file__).resolve().parent / "golden"


def _load(name):
    path = GOLDEN / name
    assert path.exists(), f"{path} missing: regenerate with tests/golden/make_golden.py"
    return np.load(path)


def test_ctc_collapse_golden(oracle_c):
    g = _load("ctc_collapse.npz")
    ids, scores = g["ids"], g["scores"]
    lines, T = ids.shape
    out = np.empty((lines, T), np.int32)
    ln = np.empty(lines, np.int32)
    sc = np.empty(lines, np.float32)
    oracle_c.oracle_ctc_collapse(np.ascontiguousarray(ids).ctypes.data, np.ascontiguousarray(scores).ctypes.data,
                                 lines, T, int(g["blank"]), out.ctypes.data, ln.ctypes.data, sc.ctypes.data)
    assert np.array_equal(out, g["out_ids"])
    assert np.array_equal(ln, g["out_len"])
    assert np.array_equal(sc, g["out_score"])  # same summation order: bit-exact


def test_classifier_golden():
    """Row argmax / max logit / 1/sum(exp) of the reference's WMMA path."""
    g = _load("classifier.npz")
    logits = g["hidden"].astype(np.float64) @ g["weight"].astype(np.float64) + g["bias"].astype(np.float64)
    ids, prob, mx = L.argmax_prob(logits)
    top2 = np.sort(logits, axis=1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-3
    assert clear.mean() > 0.9
    assert np.array_equal(ids[clear], g["ids"][clear])
    assert np.abs(mx - g["max_logit"]).max() <= 1e-3
    assert np.abs(prob - g["prob"]).max() <= 1e-4


def test_depthwise_golden_bit_exact():
    g = _load("depthwise.npz")
    names = sorted({k.split("__")[0] for k in g.files})
    assert len(names) >= 4
    for n in names:
        kh, kw, sh, sw, ph, pw, act = g[f"{n}__geom"].tolist()
        x = torch.from_numpy(g[f"{n}__x"].astype(np.float32))
        w = torch.from_numpy(g[f"{n}__w"].astype(np.float32))
        b = torch.from_numpy(g[f"{n}__bias"].astype(np.float32))
        y = L.depthwise_exact(x, w, b, (sh, sw), (ph, pw), act)
        want = torch.from_numpy(g[f"{n}__y"].astype(np.float32))
        assert torch.equal(y, want), f"{n}: max diff {(y - want).abs().max().item()}"


def test_pool_golden_bit_exact():
    g = _load("pool.npz")
    for kind, (k, s, maximum) in ((0, ((2, 2), (1, 1), True)), (1, ((3, 2), (3, 2), False))):
        x = torch.from_numpy(g[f"kind{kind}__x"].astype(np.float32))
        y = L.pool_nhwc(x, k, s, 0, maximum)
        assert torch.equal(y, torch.from_numpy(g[f"kind{kind}__y"].astype(np.float32)))


def test_preprocess_golden():
    """The numpy restatement equals the reference kernels' f32 output bit
    for bit (detector canvas with padding, BGR/RGB; ROI warp with a
    degenerate transform and crop widths below the canvas)."""
    g = _load("preprocess.npz")
    page = g["page"]
    for name in ("up_padded_rgb", "down_bgr"):
        dh, dw, ch, cw, bgr = g[f"det_{name}__geom"].tolist()
        o = OP.detector_preprocess(page, dh, dw, ch, cw, bool(bgr))
        want = g[f"det_{name}__y"]
        assert o.shape == want.shape
        assert np.array_equal(o, want), f"{name}: max diff {np.abs(o - want).max()}"
    for bgr in (0, 1):
        want = g[f"roi_bgr{bgr}__y"]
        o = OP.roi_warp(g["roi_src"], g["m_invs"], g["crop_widths"], want.shape[2], want.shape[3], bool(bgr))
        assert np.array_equal(o, want), f"roi bgr={bgr}: max diff {np.abs(o - want).max()}"
        # right of each crop's width the reference writes zeros
        for b, cw in enumerate(g["crop_widths"]):
            assert np.all(want[b, :, :, cw:] == 0)


def test_components_golden():
    """8-connected components and (left, top, width, height, area) equal
    OpenCV's connectedComponentsWithStats (the library the reference's DB
    post-processing runs on these maps), numbering included."""
    g = _load("components.npz")
    names = sorted({k.split("__")[0] for k in g.files})
    assert len(names) >= 3
    for n in names:
        labels, count, stats, _ = OC.components(g[f"{n}__bitmap"], g[f"{n}__prob"])
        assert count == g[f"{n}__stats"].shape[0]
        assert np.array_equal(labels, g[f"{n}__labels"]), n
        assert np.array_equal(stats, g[f"{n}__stats"]), n


@pytest.mark.parametrize("fixture", ["ctc_collapse.npz", "classifier.npz", "depthwise.npz", "pool.npz",
                                     "preprocess.npz", "components.npz"])
def test_golden_fixtures_are_small(fixture):
    assert (GOLDEN / fixture).stat().st_size < 512 * 1024
