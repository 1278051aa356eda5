"""Small shared helpers for the parity tests."""

import numpy as np
import torch

SEED = 20261201


def rng(seed_offset=0):
    return np.random.default_rng(SEED + seed_offset)


def f16(a) -> torch.Tensor:
    """float32 CPU tensor holding fp16-representable values."""
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.float16).to(torch.float32)


def dev(t: torch.Tensor, dtype=torch.float16) -> torch.Tensor:
    return t.to(dtype).contiguous().cuda()


def host(t: torch.Tensor) -> torch.Tensor:
    return t.float().cpu()


def rel_l2(got: torch.Tensor, want: torch.Tensor) -> float:
    got, want = got.double(), want.double()
    den = torch.linalg.vector_norm(want).item()
    return torch.linalg.vector_norm(got - want).item() / max(den, 1e-30)


def assert_close(got, want, max_abs=2e-2, rel=1e-3, what=""):
    """FP16 activation parity bar: max-abs 2e-2 and relative L2 1e-3."""
    got = got.float()
    want = want.float()
    assert got.shape == want.shape, f"{what}: shape {tuple(got.shape)} != {tuple(want.shape)}"
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    diff = (got - want).abs()
    ma = diff.max().item() if diff.numel() else 0.0
    r = rel_l2(got, want) if diff.numel() else 0.0
    where = np.unravel_index(int(diff.argmax()), tuple(diff.shape)) if diff.numel() else ()
    assert ma <= max_abs and r <= rel, (
        f"{what}: max_abs={ma:.4g} (at {where}: got {got[where].item() if diff.numel() else 0:.5g} "
        f"want {want[where].item() if diff.numel() else 0:.5g}) rel_l2={r:.3g}")


def check_decode(rec, n, oracle_c, oracle_hidden=None, margin=0.25):
    """Decoded-text parity of a LineRecognizer after rec.enqueue() of n lines.

    1. The fused vocabulary projection + argmax on the device's own hidden
       states against float64 logits from the same FP16 hidden and head
       weights: ids exact on every frame whose top-2 gap exceeds 1e-3 (at
       least 90 % of frames must be that clear), max-prob within 1e-5.
    2. The device collapse against the oracle's C collapse of the device's
       frame ids and probabilities (ctc_decode.cpp:7-51 semantics): ids,
       lengths and scores bit-exact; mean decoded length at least 8.
    3. With oracle_hidden (the CPU oracle's hidden states of the same
       lines): frames whose oracle top-2 gap exceeds `margin` (far above the
       logit error the FP16 hidden-state difference can cause) decode to the
       same id, and at least half of all frames are that clear.
    Returns (ids, lens, scores) of the device."""
    import ctypes

    ids, lens, scores = rec.results(n)
    T, H = rec.T, rec.H
    w = torch.from_numpy(rec.head.weight_host).half().double()
    b = torch.from_numpy(rec.head.bias_host).half().double()
    hidden = rec.hidden[:n].float().cpu().reshape(-1, H).double()
    logits = hidden @ w + b
    top2 = torch.topk(logits, 2, 1).values
    clear = ((top2[:, 0] - top2[:, 1]) > 1e-3).numpy()
    assert clear.mean() >= 0.9, f"only {clear.mean():.3f} of frames have a top-2 gap > 1e-3"
    want_ids = logits.argmax(1).numpy().astype(np.int32)
    want_prob = (1.0 / torch.exp(logits - top2[:, :1]).sum(1)).numpy()
    frame_ids = rec.ids[: n * T].cpu().numpy()
    frame_prob = rec.prob[: n * T].cpu().numpy()
    assert np.array_equal(frame_ids[clear], want_ids[clear])
    assert np.abs(frame_prob - want_prob).max() <= 1e-5
    o_ids = np.empty((n, T), np.int32)
    o_len = np.empty(n, np.int32)
    o_sc = np.empty(n, np.float32)
    fi = np.ascontiguousarray(frame_ids, np.int32)
    fp = np.ascontiguousarray(frame_prob, np.float32)
    oracle_c.oracle_ctc_collapse(fi.ctypes.data, fp.ctypes.data, n, T, rec.blank, o_ids.ctypes.data,
                                 o_len.ctypes.data, o_sc.ctypes.data)
    assert np.array_equal(lens, o_len)
    for k in range(n):
        assert np.array_equal(ids[k, : lens[k]], o_ids[k, : o_len[k]])
    assert np.array_equal(scores, o_sc)
    assert lens.mean() >= 8, f"degenerate decode: mean length {lens.mean()}"
    if oracle_hidden is not None:
        lo = oracle_hidden.reshape(-1, H).double() @ w + b
        t2 = torch.topk(lo, 2, 1).values
        sure = ((t2[:, 0] - t2[:, 1]) > margin).numpy()
        assert sure.mean() >= 0.5, f"only {sure.mean():.2f} of frames clear the {margin} margin"
        assert np.array_equal(frame_ids[sure], lo.argmax(1).numpy().astype(np.int32)[sure])
    del ctypes
    return ids, lens, scores
