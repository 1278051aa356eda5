"""Parity at the BASELINE configurations' own sizes, through the Model ABI v2
shell and the head C-ABI, against the CPU oracle (oracle/models.py running
the same generated graph on the same FP16 weights).

C1 (CTC head on [32, 40, 18385] logits) is covered at full size in
test_gpu_ops.py::test_logits_argmax_and_collapse. Here: C2 (the
depthwise-separable block, full [16, 48, 320, 64] input), C3 (the SVTR neck,
full [256, 40, 120] tokens), C4 (the recognizer compiled for B=512, checked
on lines at both ends of the batch), C5 (the page pipeline at 8 x 960^2:
detector map of one page against the oracle, binarize bit-exact over every
page, batch-position independence, replay determinism).
"""

import numpy as np
import pytest
import torch

from helpers import assert_close, check_decode, rng
from oracle import layers as L
from oracle import models as OM

pytestmark = pytest.mark.gpu


def _enqueue_nhwc(model, x_nhwc: torch.Tensor) -> torch.Tensor:
    stream = torch.cuda.Stream()
    out = model.output_tensor()
    model.enqueue_nhwc(x_nhwc, out, stream)
    stream.synchronize()
    return out


def test_c2_block_full_size(native, cuda):
    from ppocr_b200 import models, pipeline, workloads

    m = pipeline.CompiledModel("block_b16", cuda)
    try:
        x = workloads.c2_input(rng(40), 16)
        got = _enqueue_nhwc(m, torch.from_numpy(x).cuda()).float().cpu()
        assert native.ppocr_b200_device_error() == 0
        g, out_id = models.graph("block_b16")
        want, _ = OM.run_graph(g, x.astype(np.float32).transpose(0, 3, 1, 2), out_id)
        assert_close(got, want, what="C2 dw5x5+pw block")
    finally:
        m.close()


def test_c3_neck_full_size(native, cuda):
    from ppocr_b200 import models, pipeline, workloads

    m = pipeline.CompiledModel("neck_b256", cuda)
    try:
        tok = workloads.c3_tokens(rng(41), 256)
        got = _enqueue_nhwc(m, torch.from_numpy(tok).cuda().reshape(256, 1, 40, 120)).float().cpu()
        assert native.ppocr_b200_device_error() == 0
        g, out_id = models.graph("neck_b256")
        want, _ = OM.run_graph(g, tok.astype(np.float32).reshape(256, 1, 40, 120), out_id)
        assert_close(got, want, what="C3 SVTR neck")
    finally:
        m.close()


def test_c3_neck_partial_batch_rows_match(cuda):
    """A partial batch gives the same rows as the full batch (zero tail)."""
    from ppocr_b200 import pipeline, workloads

    m = pipeline.CompiledModel("neck_b256", cuda)
    try:
        tok = torch.from_numpy(workloads.c3_tokens(rng(42), 256)).cuda().reshape(256, 1, 40, 120)
        full = _enqueue_nhwc(m, tok).clone()
        part = _enqueue_nhwc(m, tok[:37].contiguous())
        assert torch.equal(part[:37], full[:37])
    finally:
        m.close()


def test_c4_recognizer_b512_ends_of_batch(native, cuda, oracle_c):
    """The B=512 bench shape through the whole line path (model, fused head,
    device collapse): every line's decoded text against the oracle head on
    the device hidden states, and lines at both ends of the batch against the
    oracle graph (built for 4 lines, same seeded weights): hidden states at
    the north-star bar, clear frames' ids end to end."""
    from ppocr_b200 import models, modelgen, pipeline, workloads

    rec = pipeline.LineRecognizer("rec_b512", cuda)
    try:
        x = workloads.c4_lines(rng(43), 512)
        rec.enqueue(torch.from_numpy(x).cuda())
        rec.stream.synchronize()
        assert native.ppocr_b200_device_error() == 0
        got = rec.hidden.float().cpu()
        pick = [0, 1, 510, 511]
        g, out_id = modelgen.build_recognizer(models.spec("recognizer"), 4, models.SEED)
        want, _ = OM.run_graph(g, x[pick].astype(np.float32).transpose(0, 3, 1, 2), out_id)
        assert_close(got[pick], want, what="C4 recognizer hidden, lines 0, 1, 510, 511")
        check_decode(rec, 512, oracle_c)
        # End to end on the picked lines: the oracle's hidden states decode
        # to the device's ids on every frame with a clear margin.
        w = torch.from_numpy(rec.head.weight_host).half().double()
        b = torch.from_numpy(rec.head.bias_host).half().double()
        lo = want.reshape(-1, rec.H).double() @ w + b
        t2 = torch.topk(lo, 2, 1).values
        sure = ((t2[:, 0] - t2[:, 1]) > 0.25).numpy()
        frame_ids = rec.ids.cpu().numpy().reshape(512, rec.T)[pick].reshape(-1)
        assert sure.mean() >= 0.5
        assert np.array_equal(frame_ids[sure], lo.argmax(1).numpy().astype(np.int32)[sure])
    finally:
        rec.close()


def test_c5_page_pipeline_full_size(native, cuda):
    from ppocr_b200 import models, modelgen, pipeline, workloads

    pp = pipeline.PagePipeline(device=cuda)
    try:
        pages, crops = workloads.c5_pages(rng(44))
        dp, dc = torch.from_numpy(pages).cuda(), torch.from_numpy(crops).cuda()
        pp.enqueue(dp, dc)
        pp.stream.synchronize()
        assert native.ppocr_b200_device_error() == 0
        prob = pp.prob.cpu().clone()
        bitmap = pp.bitmap.cpu().clone()
        ids, lens, scores = pp.rec.results(512)
        assert prob.shape == (8, 1, 960, 960) and prob.dtype == torch.float32
        assert torch.isfinite(prob).all() and prob.min() >= 0 and prob.max() <= 1
        # DB binarize over all eight maps, bit-exact (cv::compare CMP_GT).
        assert np.array_equal(bitmap.numpy().ravel(), L.binarize(prob.numpy().ravel(), pp.thresh))
        # Page 3's map against the oracle (detector graph built for one page,
        # same seeded weights).
        g, out_id = modelgen.build_detector(models.spec("detector"), 1, 960, models.SEED)
        want, _ = OM.run_graph(g, pages[3:4].astype(np.float32).transpose(0, 3, 1, 2), out_id)
        assert_close(prob[3:4], want, what="C5 detector map, page 3")
        away = (want - pp.thresh).abs() > 2e-3
        assert torch.equal(bitmap[3:4][away], torch.from_numpy(L.binarize(want.numpy(), pp.thresh))[away])
        # Page order reversed: every map moves with its page, bit for bit;
        # the recognizer output replays identically.
        pp.enqueue(dp.flip(0).contiguous(), dc)
        pp.stream.synchronize()
        assert torch.equal(pp.prob.cpu(), prob.flip(0))
        ids2, lens2, scores2 = pp.rec.results(512)
        assert np.array_equal(ids, ids2) and np.array_equal(lens, lens2) and np.array_equal(scores, scores2)
        # End to end from pinned host memory (copies overlapped with the
        # detector and recognizer on side streams): the same maps and tokens,
        # twice in a row (the second call reuses the staging buffers), and
        # with fewer crops than the compiled batch.
        ph, ch = torch.from_numpy(pages).pin_memory(), torch.from_numpy(crops).pin_memory()
        bm_h = torch.zeros(8, 1, 960, 960, dtype=torch.uint8).pin_memory()
        ids_h = torch.zeros(512, pp.rec.T, dtype=torch.int32).pin_memory()
        len_h = torch.zeros(512, dtype=torch.int32).pin_memory()
        sc_h = torch.zeros(512, dtype=torch.float32).pin_memory()
        for _ in range(2):
            bm_h.zero_()
            ids_h.zero_()
            pp.enqueue_host(ph, ch, bm_h, ids_h, len_h, sc_h)
            pp.stream.synchronize()
            assert torch.equal(bm_h, bitmap)
            assert np.array_equal(ids_h.numpy(), ids) and np.array_equal(len_h.numpy(), lens)
            assert np.array_equal(sc_h.numpy(), scores)
        len_h.fill_(-1)
        pp.enqueue_host(ph, ch[:100], bm_h, ids_h, len_h, sc_h)
        pp.stream.synchronize()
        assert np.array_equal(len_h[:100].numpy(), lens[:100]) and (len_h[100:] == -1).all()
        assert native.ppocr_b200_device_error() == 0
    finally:
        pp.close()
