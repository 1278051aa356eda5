"""Whole-graph parity on the B200 through the Model ABI v2 shell
(include/ppocr_b200_model_abi.h) against the CPU oracle running the same
generated graph (oracle/models.py), plus the reference's replay and
partial-batch contracts (native/tests/tools/compiled_memory_smoke.cpp:
91-92 bit-identical replay; model_library.cu:15-20 zero tail)."""

import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_close, check_decode, rng
from oracle import layers as L
from oracle import models as OM

pytestmark = pytest.mark.gpu


def _input(batch, h, w, seed):
    return rng(seed).uniform(-1, 1, (batch, 3, h, w)).astype(np.float32)


def _run_f32(model, x):
    from ppocr_b200 import pipeline  # noqa: F401

    stream = torch.cuda.Stream()
    dx = torch.from_numpy(x).cuda()
    out = model.output_tensor()
    model.enqueue_f32(dx, out, stream)
    stream.synchronize()
    return out


@pytest.fixture(scope="module")
def rec2(cuda):
    from ppocr_b200 import pipeline

    m = pipeline.CompiledModel("rec_b2", cuda)
    yield m
    m.close()


def test_recognizer_abi_matches_oracle(native, rec2):
    from ppocr_b200 import models

    x = _input(2, 48, 320, 1)
    got = _run_f32(rec2, x).float().cpu()
    g, out_id = models.graph("rec_b2")
    want, _ = OM.run_graph(g, x, out_id)
    assert native.ppocr_b200_device_error() == 0
    assert got.shape == want.shape
    # 30 fp16-stored layers: per-element rounding flips propagate; the
    # whole-graph bar is the north-star one (max-abs 2e-2, rel-L2 1e-3).
    assert_close(got, want, what="recognizer rec_b2 hidden")


def test_recognizer_replay_bit_identical_and_nhwc_entry(rec2):
    x = _input(2, 48, 320, 2)
    a = _run_f32(rec2, x).clone()
    b = _run_f32(rec2, x).clone()
    assert torch.equal(a, b)
    # FP16 NHWC entry point on the same images gives the same output.
    stream = torch.cuda.Stream()
    xh = torch.from_numpy(x).cuda().half().permute(0, 2, 3, 1).contiguous()
    out = rec2.output_tensor()
    rec2.enqueue_nhwc(xh, out, stream)
    stream.synchronize()
    assert torch.equal(out, a)


def test_first_enqueue_equals_replay(cuda):
    """The first enqueue (eager warm-up + capture + launch) of a fresh handle
    must give the same output as later graph replays, even though the staged
    channels-last input shares arena storage with later tensors."""
    from ppocr_b200 import pipeline

    m = pipeline.CompiledModel("rec_b2", cuda)
    try:
        x = _input(2, 48, 320, 9)
        first = _run_f32(m, x).clone()
        second = _run_f32(m, x).clone()
        assert torch.equal(first, second)
    finally:
        m.close()


def test_timed_out_wait_fails_next_enqueue(native, rec2):
    """A bounded wait that ran out during a graph replay (its code stored in
    the library's error word as the kernel would store it) makes the next
    enqueue of the handle fail with the code; the word is then clear."""
    from ppocr_b200.capi import NativeError

    x = _input(2, 48, 320, 6)
    _run_f32(rec2, x)
    assert native.ppocr_b200_test_store_error_code(0, 5) == 0, native.ppocr_b200_last_error()
    _run_f32(rec2, x)  # this replay's copy of the word sees the code
    with pytest.raises(NativeError, match=r"kernel wait timed out in the previous batch \(code 5\)"):
        _run_f32(rec2, x)
    assert native.ppocr_b200_device_error() == 0
    _run_f32(rec2, x)  # the handle keeps working


def test_recognizer_partial_batch(rec2):
    x = _input(2, 48, 320, 3)
    full = _run_f32(rec2, x).clone()
    stream = torch.cuda.Stream()
    dx = torch.from_numpy(x[:1].copy()).cuda()
    out = rec2.output_tensor()
    out.fill_(7)
    rec2.enqueue_f32(dx, out, stream)
    stream.synchronize()
    assert torch.equal(out[0], full[0])
    assert torch.all(out[1] == 7)  # rows past `batch` are not written


def test_recognizer_rejects_bad_batch(rec2):
    from ppocr_b200.capi import NativeError

    stream = torch.cuda.Stream()
    dx = torch.zeros(3, 3, 48, 320, device="cuda")
    out = rec2.output_tensor()
    with pytest.raises(NativeError, match="Invalid compiled model input/batch"):
        rec2.enqueue_f32(dx, out, stream)


def test_detector_abi_matches_oracle_and_binarize(native, cuda):
    from ppocr_b200 import models, pipeline

    m = pipeline.CompiledModel("det_b1_s128", cuda)
    try:
        x = _input(1, 128, 128, 4)
        got = _run_f32(m, x).float().cpu()
        g, out_id = models.graph("det_b1_s128")
        want, _ = OM.run_graph(g, x, out_id)
        assert got.dtype == torch.float32 and got.shape == (1, 1, 128, 128)
        assert_close(got, want, what="detector map det_b1_s128")
        # binarize on device vs oracle, bit-exact away from the threshold
        dprob = got.cuda().contiguous()
        bmap = torch.empty(dprob.numel(), dtype=torch.uint8, device="cuda")
        assert native.ppocr_b200_binarize(ctypes.c_void_p(dprob.data_ptr()), ctypes.c_void_p(bmap.data_ptr()),
                                          dprob.numel(), 0.3, None) == 0
        torch.cuda.synchronize()
        got_map = bmap.cpu().numpy()
        want_map = L.binarize(want.numpy().ravel(), 0.3)
        away = np.abs(want.numpy().ravel() - 0.3) > 2e-3
        assert np.array_equal(got_map[away], want_map[away])
    finally:
        m.close()


def test_line_recognizer_tokens(cuda, oracle_c):
    """Model + fused head + device collapse vs the oracle's tokens: frame ids,
    probabilities, collapsed ids / lengths / scores, and the end-to-end
    decode from the oracle's own hidden states on clear frames."""
    from ppocr_b200 import models, pipeline

    rec = pipeline.LineRecognizer("rec_b2", cuda)
    try:
        x = _input(2, 48, 320, 5)
        xh = torch.from_numpy(x).cuda().half().permute(0, 2, 3, 1).contiguous()
        rec.enqueue(xh)
        g, out_id = models.graph("rec_b2")
        want_hidden, _ = OM.run_graph(g, x, out_id)
        ids, lens, scores = check_decode(rec, 2, oracle_c, want_hidden)
        assert lens.shape == (2,) and np.all(lens <= rec.T)
    finally:
        rec.close()


def test_line_stream_matches_serial(cuda):
    """Double-buffered host stream (copy of batch k+1 during batch k) decodes
    every batch, short ones included, exactly as a serial copy + enqueue."""
    from ppocr_b200 import pipeline

    rec = pipeline.LineRecognizer("rec_b2", cuda)
    try:
        sizes = [2, 1, 2, 2, 1]
        batches = [torch.from_numpy(rng(40 + k).uniform(-1, 1, (n, 48, 320, 3)).astype(np.float16)).pin_memory()
                   for k, n in enumerate(sizes)]
        want = []
        for b in batches:
            rec.enqueue(b.cuda())
            want.append(rec.results(b.shape[0]))
        outs = [(torch.full((2, rec.T), -1, dtype=torch.int32).pin_memory(),
                 torch.full((2,), -1, dtype=torch.int32).pin_memory(),
                 torch.full((2,), -1.0, dtype=torch.float32).pin_memory()) for _ in sizes]
        stream = pipeline.LineStream(rec)
        stream.enqueue(batches, outs)
        rec.stream.synchronize()
        for (ids, lens, scores), (wi, wl, ws), n in zip(outs, want, sizes):
            assert np.array_equal(ids[:n].numpy(), wi) and np.array_equal(lens[:n].numpy(), wl)
            assert np.array_equal(scores[:n].numpy(), ws)
            assert np.all(lens[n:].numpy() == -1)
    finally:
        rec.close()


def test_model_stream_matches_serial(cuda):
    """ModelStream (input copy of batch k+1 and output copy of batch k-1 on
    their own streams while batch k runs) returns every batch's output, short
    batches included, exactly as a serial copy + enqueue + read back."""
    from ppocr_b200 import pipeline

    model = pipeline.CompiledModel("neck_b256", cuda)
    try:
        sizes = [256, 100, 256, 7, 256]
        batches = [torch.from_numpy(rng(80 + k).standard_normal((n, 1, 40, 120)).astype(np.float16)).pin_memory()
                   for k, n in enumerate(sizes)]
        stream = torch.cuda.Stream(cuda)
        want = []
        out = model.output_tensor()
        for b in batches:
            model.enqueue_nhwc(b.to(cuda), out, stream)
            stream.synchronize()
            want.append(out[: b.shape[0]].cpu().clone())
        outs = [torch.full(tuple(out.shape), -1.0, dtype=out.dtype).pin_memory() for _ in sizes]
        ms = pipeline.ModelStream(model, stream)
        ms.enqueue(batches, outs)
        ms.join(stream)
        stream.synchronize()
        for got, w, n in zip(outs, want, sizes):
            assert torch.equal(got[:n], w)
            assert torch.all(got[n:] == -1)
    finally:
        model.close()


def test_runtime_fusions_and_split_back(native, cuda):
    """The Runtime's speculative fusions (depthwise + pointwise block, lateral
    1x1 + FPN resize-add, DB-head transposed-conv pair) on a chained test
    graph: with nothing else reading the intermediates each pair runs fused
    (its second slot an empty "fused" placeholder); in the twin graph a later
    op reads every intermediate, so every pair splits back into its two ops
    in place. The chain output is bit-identical both ways and within the
    fp16 bar of the oracle."""
    from ppocr_b200 import models, pipeline

    x = _input(2, 16, 16, 77)
    outs = {}
    for name in ("probe_fused", "probe_split"):
        m = pipeline.CompiledModel(name, cuda)
        try:
            names = m.lib.op_names(m.handle)
            outs[name] = _run_f32(m, x).cpu()
        finally:
            m.close()
        fused = {"dwpw_block", "gemm_resize_add", "deconv_db_tail"}
        if name == "probe_fused":
            assert fused <= set(names) and names.count("fused") == 3, names
        else:
            assert not fused & set(names) and "fused" not in names, names
            assert {"depthwise", "resize_add_nhwc", "deconv_tc", "deconv"} <= set(names), names
    assert torch.equal(outs["probe_fused"].view(torch.int16), outs["probe_split"].view(torch.int16))
    g, out_id = models.graph("probe_fused")
    want, _ = OM.run_graph(g, x, out_id)
    assert_close(outs["probe_fused"], want, what="fusion probe")
    assert native.ppocr_b200_device_error() == 0
