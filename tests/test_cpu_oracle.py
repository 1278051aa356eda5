"""CPU tests: the oracle pinned to the reference's own golden vectors and to
the reference's compiled CTC decoder; no GPU needed."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import rng
from oracle import layers as L

REPO = Path(__file__).resolve().parent.parent
REF_CTC = REPO / "oracle" / "_ref" / "libref_ctc.so"

# native/tests/tools/ctc_smoke.cpp:21-38
GOLDEN_CHARS = ["blank", "a", "b", "c", " "]
GOLDEN_IDS = [0, 1, 1, 0, 2, 2, 3, 0, 2, 0, 2, 2, 0, 1, 1, 3]
GOLDEN_SCORES = [1.0, 0.8, 0.7, 1.0, 0.7, 0.6, 0.9, 1.0, 0.5, 1.0, 0.6, 0.4, 1.0, 0.9, 0.8, 0.7]
GOLDEN_TEXT = ["abc", "bbac"]
GOLDEN_MEAN = [0.8, 0.675]


def collapse(oracle_c, ids, scores, lines, T, blank=0):
    ids = np.ascontiguousarray(ids, np.int32)
    sc = None if scores is None else np.ascontiguousarray(scores, np.float32)
    out = np.empty((lines, T), np.int32)
    ln = np.empty(lines, np.int32)
    s = np.empty(lines, np.float32)
    oracle_c.oracle_ctc_collapse(ids.ctypes.data, None if sc is None else sc.ctypes.data, lines, T, blank,
                                 out.ctypes.data, ln.ctypes.data, s.ctypes.data)
    return out, ln, s


def test_oracle_collapse_golden(oracle_c):
    out, ln, s = collapse(oracle_c, GOLDEN_IDS, GOLDEN_SCORES, 2, 8)
    texts = ["".join(GOLDEN_CHARS[i] for i in out[r, : ln[r]]) for r in range(2)]
    assert texts == GOLDEN_TEXT
    assert abs(s[0] - GOLDEN_MEAN[0]) < 1e-6 and abs(s[1] - GOLDEN_MEAN[1]) < 1e-6


def test_oracle_collapse_edge_cases(oracle_c):
    # all blank -> nothing kept, score 0; repeats separated by blank are kept
    out, ln, s = collapse(oracle_c, [0, 0, 0, 0], [0.5] * 4, 1, 4)
    assert ln[0] == 0 and s[0] == 0.0 and np.all(out == -1)
    out, ln, s = collapse(oracle_c, [3, 0, 3, 3], None, 1, 4)
    assert out[0, :2].tolist() == [3, 3] and ln[0] == 2 and s[0] == 1.0
    # out-of-vocabulary ids are kept (the reference prints them as "<id>")
    out, ln, _ = collapse(oracle_c, [99999, -5], None, 1, 2)
    assert out[0].tolist() == [99999, -5]


@pytest.fixture(scope="module")
def ref_ctc():
    if not REF_CTC.exists():
        pytest.skip("reference CTC decoder not built (needs the reference sources)")
    lib = ctypes.CDLL(str(REF_CTC))
    P = ctypes.c_void_p
    lib.ref_ctc_decode_batch.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P]
    lib.ref_ctc_decode_text.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                        ctypes.c_char_p, ctypes.c_int, P]
    return lib


def test_reference_decoder_golden(ref_ctc):
    ids = np.array(GOLDEN_IDS, np.int32)
    sc = np.array(GOLDEN_SCORES, np.float32)
    buf = ctypes.create_string_buffer(256)
    scores = np.empty(2, np.float32)
    assert ref_ctc.ref_ctc_decode_text(ids.ctypes.data, sc.ctypes.data, 2, 8, "\n".join(GOLDEN_CHARS).encode(), 0,
                                       buf, 256, scores.ctypes.data) == 0
    assert buf.value.decode().split("\n") == GOLDEN_TEXT


@pytest.mark.parametrize("with_scores", [True, False])
def test_oracle_matches_compiled_reference(oracle_c, ref_ctc, with_scores):
    r = rng(40)
    lines, T = 2000, 40
    ids = r.integers(0, 8, (lines, T)).astype(np.int32)
    ids[::7] = 0
    ids[1::11] = r.integers(0, 18385, (len(ids[1::11]), T))
    sc = r.random((lines, T)).astype(np.float32) if with_scores else None
    o_ids, o_len, o_s = collapse(oracle_c, ids, sc, lines, T)
    r_ids = np.empty((lines, T), np.int32)
    r_len = np.empty(lines, np.int32)
    r_s = np.empty(lines, np.float32)
    assert ref_ctc.ref_ctc_decode_batch(ids.ctypes.data, None if sc is None else sc.ctypes.data, lines, T, 0,
                                        r_ids.ctypes.data, r_len.ctypes.data, r_s.ctypes.data) == 0
    assert np.array_equal(o_ids, r_ids)
    assert np.array_equal(o_len, r_len)
    assert np.array_equal(o_s, r_s)  # same float summation order -> bit-exact


def test_oracle_argmax_prob(oracle_c):
    r = rng(41)
    rows, V = 64, 18385
    logits = r.standard_normal((rows, V)).astype(np.float16)
    logits[3, 10] = logits[3, 20] = 9.0  # tie -> lowest id
    ids = np.empty(rows, np.int32)
    prob = np.empty(rows, np.float32)
    mx = np.empty(rows, np.float32)
    oracle_c.oracle_argmax_prob(logits.ctypes.data, rows, V, ids.ctypes.data, prob.ctypes.data, mx.ctypes.data, 2)
    w_ids, w_prob, w_max = L.argmax_prob(logits.astype(np.float32))
    assert ids[3] == 10
    assert np.array_equal(ids, w_ids)
    assert np.allclose(prob, w_prob, rtol=1e-6, atol=1e-7)
    assert np.array_equal(mx, w_max)


def test_depthwise_oracle_orders_taps_like_reference():
    """The exact-order depthwise restatement agrees with torch's conv to fp32
    rounding noise (its bit-exactness is pinned on the GPU box)."""
    r = rng(42)
    x = L.rh(torch.from_numpy(r.uniform(-1, 1, (1, 9, 11, 16)).astype(np.float32)))
    w = L.rh(torch.from_numpy(r.standard_normal((16, 3, 3)).astype(np.float32)))
    b = L.rh(torch.from_numpy(r.normal(0, 0.1, 16).astype(np.float32)))
    a = L.depthwise_exact(x, w, b, (2, 1), (1, 1), 1)
    c = L.conv_nhwc(x, w, b, (2, 1), (1, 1), 16, 1)
    assert (a - c).abs().max().item() <= 2 ** -9


def test_binarize_oracle():
    p = np.array([0.3, np.nextafter(np.float32(0.3), 1), 0.29, 1.0, 0.0], np.float32)
    assert L.binarize(p, 0.3).tolist() == [0, 255, 0, 255, 0]
