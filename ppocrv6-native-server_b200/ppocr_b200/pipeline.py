"""Line recognizer and page pipeline over the C-ABI, one replica per GPU.

Mirrors the reference's worker flow (native/src/recognition/
recognition_worker.cpp:700-746: enqueue the compiled model, launch the
classifier, collapse; native/src/full_page/full_page_worker.cpp:361-497 for
pages) with every step on the device: the model graph, the fused vocabulary
projection + argmax, and the CTC collapse. torch provides device memory and
streams only.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import torch

from . import capi, models, modelgen


def _p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class CompiledModel:
    """One compiled shape: weights (shared), scratch, a handle, CUDA graph."""

    def __init__(self, name: str, device: torch.device, weights_ptr: int | None = None):
        self.name = name
        self.device = device
        self.lib = capi.ModelLibrary(models.library_path(name))
        info = self.lib.info
        self.input_shape = tuple(info.input_shape)
        self.output_shape = tuple(info.output_shape[: info.output_rank])
        self.output_bytes = info.output_element_bytes
        with torch.cuda.device(device):
            self._owns_weights = weights_ptr is None
            self.weights = weights_ptr or self.lib.load_weights(models.ensure_weights(name))
            self.scratch = torch.empty(info.scratch_bytes, dtype=torch.uint8, device=device)
            self.handle = self.lib.create(self.weights, self.scratch.data_ptr(), info.scratch_bytes)

    def output_tensor(self) -> torch.Tensor:
        dtype = torch.float16 if self.output_bytes == 2 else torch.float32
        return torch.empty(self.output_shape, dtype=dtype, device=self.device)

    def enqueue_nhwc(self, x: torch.Tensor, out: torch.Tensor, stream: torch.cuda.Stream) -> None:
        self.lib.enqueue_nhwc_f16(self.handle, x.data_ptr(), out.data_ptr(), x.shape[0],
                                  ctypes.c_void_p(stream.cuda_stream))

    def enqueue_f32(self, x: torch.Tensor, out: torch.Tensor, stream: torch.cuda.Stream) -> None:
        self.lib.enqueue(self.handle, x.data_ptr(), out.data_ptr(), x.shape[0],
                         ctypes.c_void_p(stream.cuda_stream))

    def close(self) -> None:
        if self.handle:
            self.lib.destroy(self.handle)
            self.handle = None
        if self._owns_weights and self.weights:
            torch.cuda.synchronize(self.device)
            capi.load().ppocr_b200_device_free(ctypes.c_void_p(self.weights))
            self.weights = None


class Classifier:
    """CTC head weights resident on the device in the packed layout."""

    def __init__(self, hidden: int, vocab: int, device: torch.device, seed: int = models.SEED):
        w, b = models.head_weights(hidden, vocab, seed)
        self.hidden, self.vocab = hidden, vocab
        self.weight_host = w
        self.bias_host = b
        self.device = device
        self.weight = torch.from_numpy(w).to(torch.float16).to(device)
        self.bias = torch.from_numpy(b).to(torch.float16).to(device)
        self.packed = torch.empty(vocab, hidden, dtype=torch.float16, device=device)
        lib = capi.load()
        capi.check(lib.ppocr_b200_classifier_pack(_p(self.weight), _p(self.packed), hidden, vocab,
                                                  ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)))


class LineRecognizer:
    """Compiled recognizer shape + head + device collapse on one GPU."""

    def __init__(self, name: str, device: torch.device | str = "cuda:0"):
        self.device = torch.device(device)
        self.model = CompiledModel(name, self.device)
        spec = models.spec("recognizer")
        self.batch = self.model.input_shape[0]
        _, self.T, self.H = self.model.output_shape
        self.vocab = spec["vocab"]
        self.blank = spec["blank"]
        with torch.cuda.device(self.device):
            self.head = Classifier(self.H, self.vocab, self.device)
            self.stream = torch.cuda.Stream(self.device)
            rows = self.batch * self.T
            tiles = (self.vocab + 255) // 256
            self.hidden = self.model.output_tensor()
            self.part_id = torch.empty(rows * tiles, dtype=torch.int32, device=self.device)
            self.part_max = torch.empty(rows * tiles, dtype=torch.float32, device=self.device)
            self.part_sum = torch.empty(rows * tiles, dtype=torch.float32, device=self.device)
            self.ids = torch.empty(rows, dtype=torch.int32, device=self.device)
            self.prob = torch.empty(rows, dtype=torch.float32, device=self.device)
            self.maxl = torch.empty(rows, dtype=torch.float32, device=self.device)
            self.out_ids = torch.empty(self.batch, self.T, dtype=torch.int32, device=self.device)
            self.out_len = torch.empty(self.batch, dtype=torch.int32, device=self.device)
            self.out_score = torch.empty(self.batch, dtype=torch.float32, device=self.device)
        self.lib = capi.load()

    def enqueue(self, x_nhwc: torch.Tensor) -> None:
        """Full forward of an FP16 NHWC batch on self.stream (asynchronous)."""
        self.model.enqueue_nhwc(x_nhwc, self.hidden, self.stream)
        self.enqueue_head(x_nhwc.shape[0])

    def enqueue_head(self, n: int) -> None:
        """Vocabulary projection + argmax/softmax-max + collapse of the first
        n lines of self.hidden (asynchronous, on self.stream)."""
        s = ctypes.c_void_p(self.stream.cuda_stream)
        rows = n * self.T
        capi.check(self.lib.ppocr_b200_classifier_run_packed(
            _p(self.hidden), _p(self.head.packed), _p(self.head.bias), _p(self.ids), _p(self.prob), _p(self.maxl),
            rows, self.H, self.vocab, _p(self.part_id), _p(self.part_max), _p(self.part_sum), 1, s))
        capi.check(self.lib.ppocr_b200_ctc_collapse(
            _p(self.ids), _p(self.prob), n, self.T, self.blank, _p(self.out_ids), _p(self.out_len),
            _p(self.out_score), s))

    def results(self, n: int):
        """Host copy of (ids [n,T], lengths [n], scores [n]) after synchronizing."""
        self.stream.synchronize()
        return (self.out_ids[:n].cpu().numpy(), self.out_len[:n].cpu().numpy(),
                self.out_score[:n].cpu().numpy())

    def close(self) -> None:
        self.model.close()


class LineStream:
    """Host batches in, decoded lines out, with the host->device copy of batch
    k+1 running on a copy stream while the recognizer works on batch k.

    The reference's worker copies each batch and then enqueues the model on
    one stream (recognition_worker.cpp:700-746), so the copy and the forward
    take turns; here two device staging buffers alternate: batch k+1 is
    copied into one while batch k is read from the other, and a copy into a
    buffer waits for the forward that last read it. Results go back on the
    recognizer's stream right after each batch's collapse.
    """

    def __init__(self, rec: LineRecognizer):
        self.rec = rec
        with torch.cuda.device(rec.device):
            self.copy_stream = torch.cuda.Stream(rec.device)
            b, c, h, w = rec.model.input_shape
            self.stage = [torch.empty(b, h, w, c, dtype=torch.float16, device=rec.device) for _ in range(2)]
            self.copied = [torch.cuda.Event() for _ in range(2)]
            self.consumed = [torch.cuda.Event() for _ in range(2)]
        self._used = [False, False]

    def enqueue(self, batches, outputs) -> None:
        """Asynchronous. batches[k]: pinned FP16 NHWC host tensor [n_k, 48,
        W, 3] (n_k <= the compiled batch); outputs[k]: pinned host tensors
        (ids [>=n_k, T] int32, lengths [>=n_k] int32, scores [>=n_k] f32)
        written once the recognizer's stream reaches them. Copies start after
        all work already queued on the recognizer's stream."""
        if len(batches) != len(outputs):
            raise ValueError("one output triple per batch")
        rec = self.rec
        self.copy_stream.wait_stream(rec.stream)

        def copy_in(k: int) -> None:
            s = k % 2
            if self._used[s]:
                self.copy_stream.wait_event(self.consumed[s])
            with torch.cuda.stream(self.copy_stream):
                self.stage[s][: batches[k].shape[0]].copy_(batches[k], non_blocking=True)
                self.copied[s].record(self.copy_stream)

        if batches:
            copy_in(0)
        for k, host in enumerate(batches):
            s = k % 2
            if k + 1 < len(batches):
                copy_in(k + 1)
            n = host.shape[0]
            rec.stream.wait_event(self.copied[s])
            rec.enqueue(self.stage[s][:n])
            self.consumed[s].record(rec.stream)
            self._used[s] = True
            ids, lens, scores = outputs[k]
            with torch.cuda.stream(rec.stream):
                ids[:n].copy_(rec.out_ids[:n], non_blocking=True)
                lens[:n].copy_(rec.out_len[:n], non_blocking=True)
                scores[:n].copy_(rec.out_score[:n], non_blocking=True)


class ModelStream:
    """Host batches in, host outputs out, for any compiled model, with both
    copies off the model's critical path: the host->device copy of batch k+1
    runs on one copy stream and the device->host copy of batch k-1 on
    another while the model works on batch k.

    Two device input buffers and two device output buffers alternate. A copy
    into an input buffer waits for the forward that last read it; a forward
    into an output buffer waits for the device->host copy that last read it.
    The reference's workers copy, enqueue and read back on one stream
    (recognition_worker.cpp:700-746), so the three take turns; LineStream
    overlaps only the input copy (the recognizer's outputs are small).
    """

    def __init__(self, model: CompiledModel, stream: torch.cuda.Stream | None = None):
        self.model = model
        dev = model.device
        with torch.cuda.device(dev):
            self.stream = stream if stream is not None else torch.cuda.Stream(dev)
            self.h2d = torch.cuda.Stream(dev)
            self.d2h = torch.cuda.Stream(dev)
            self.out = [model.output_tensor() for _ in range(2)]
            self.copied, self.consumed, self.produced, self.drained = (
                [torch.cuda.Event() for _ in range(2)] for _ in range(4))
        self.stage: list[torch.Tensor | None] = [None, None]
        self._in_used = [False, False]
        self._out_used = [False, False]

    def _stage(self, s: int, host: torch.Tensor) -> torch.Tensor:
        buf = self.stage[s]
        if buf is None or buf.shape[1:] != host.shape[1:] or buf.dtype != host.dtype or buf.shape[0] < host.shape[0]:
            if self._in_used[s]:
                self.consumed[s].synchronize()
            buf = torch.empty((self.model.input_shape[0],) + tuple(host.shape[1:]), dtype=host.dtype,
                              device=self.model.device)
            self.stage[s] = buf
        return buf

    def enqueue(self, batches, outputs) -> None:
        """Asynchronous. batches[k]: pinned FP16 NHWC host tensor of n_k <=
        the compiled batch images; outputs[k]: pinned host tensor receiving
        the first n_k output rows. Work starts after everything already
        queued on `self.stream`; join() orders a stream after the last
        device->host copy."""
        if len(batches) != len(outputs):
            raise ValueError("one output per batch")
        self.h2d.wait_stream(self.stream)

        def copy_in(k: int) -> None:
            s = k % 2
            buf = self._stage(s, batches[k])
            if self._in_used[s]:
                self.h2d.wait_event(self.consumed[s])
            with torch.cuda.stream(self.h2d):
                buf[: batches[k].shape[0]].copy_(batches[k], non_blocking=True)
                self.copied[s].record(self.h2d)

        if batches:
            copy_in(0)
        for k, host in enumerate(batches):
            s = k % 2
            if k + 1 < len(batches):
                copy_in(k + 1)
            n = host.shape[0]
            self.stream.wait_event(self.copied[s])
            if self._out_used[s]:
                self.stream.wait_event(self.drained[s])
            self.model.enqueue_nhwc(self.stage[s][:n], self.out[s], self.stream)
            self.consumed[s].record(self.stream)
            self.produced[s].record(self.stream)
            self._in_used[s] = self._out_used[s] = True
            self.d2h.wait_event(self.produced[s])
            with torch.cuda.stream(self.d2h):
                outputs[k][:n].copy_(self.out[s][:n], non_blocking=True)
                self.drained[s].record(self.d2h)

    def join(self, stream: torch.cuda.Stream) -> None:
        """Orders `stream` after every copy enqueued so far."""
        stream.wait_stream(self.d2h)


class PagePipeline:
    """Full-page path on one GPU: detector graph -> DB binarize -> recognizer
    over the page's line crops -> fused head -> device collapse, all on one
    stream (reference: full_page_worker.cpp:361-497 runs detection, then
    recognition of the warped crops; the crops here are given, the ROI warp
    being outside this path)."""

    def __init__(self, detector: str = "det_b8", recognizer: str = "rec_b512",
                 device: torch.device | str = "cuda:0", thresh: float | None = None):
        self.device = torch.device(device)
        self.rec = LineRecognizer(recognizer, self.device)
        self.det = CompiledModel(detector, self.device)
        self.stream = self.rec.stream
        self.thresh = models.spec("detector")["thresh"] if thresh is None else thresh
        self.pages = self.det.input_shape[0]
        self.size = self.det.input_shape[2]
        with torch.cuda.device(self.device):
            self.prob = self.det.output_tensor()
            self.bitmap = torch.empty(self.prob.shape, dtype=torch.uint8, device=self.device)
        self.lib = capi.load()

    def enqueue(self, pages_nhwc: torch.Tensor, crops_nhwc: torch.Tensor) -> None:
        """pages FP16 NHWC [<=pages, S, S, 3], crops FP16 NHWC [<=lines, 48, 320, 3]."""
        self.det.enqueue_nhwc(pages_nhwc, self.prob, self.stream)
        n = pages_nhwc.shape[0] * self.size * self.size
        capi.check(self.lib.ppocr_b200_binarize(_p(self.prob), _p(self.bitmap), n, self.thresh,
                                                ctypes.c_void_p(self.stream.cuda_stream)))
        self.rec.enqueue(crops_nhwc)

    def enqueue_host(self, pages_h: torch.Tensor, crops_h: torch.Tensor, bitmap_h: torch.Tensor,
                     ids_h: torch.Tensor, len_h: torch.Tensor, score_h: torch.Tensor) -> None:
        """One page batch end to end from pinned host memory, asynchronous on
        the pipeline's stream: pages in, binary maps and decoded lines out.

        The reference's full-page worker copies, detects, reads the map back
        and then recognizes in turn (full_page_worker.cpp:361-497,
        detection_worker.cpp:402-405). Here one copy stream brings the first
        half of the pages, the second half and then the crops in that order;
        the detector runs on each half of the pages as soon as it lands
        (a half-batch compiled shape, `half_detector`, sharing the detector's
        weights), so the second half's copy and the crops' copy overlap
        detection. The binary maps go back on a second copy stream during the
        recognizer. The batch is complete when the pipeline's stream passes
        every copy (an event recorded on it after this call marks the end of
        the whole batch); a later call's copies start after this batch.
        bitmap_h: uint8 [>=pages, 1, S, S]; ids_h int32 [>=lines, T];
        len_h int32 [>=lines]; score_h f32 [>=lines]."""
        if not hasattr(self, "_h2d"):
            with torch.cuda.device(self.device):
                self._h2d = torch.cuda.Stream(self.device)
                self._d2h = torch.cuda.Stream(self.device)
                self._stage_pages = torch.empty(self.pages, self.size, self.size, 3, dtype=torch.float16,
                                                device=self.device)
                b, c, h, w = self.rec.model.input_shape
                self._stage_crops = torch.empty(b, h, w, c, dtype=torch.float16, device=self.device)
                self._half_in = [torch.cuda.Event(), torch.cuda.Event()]
                self._crops_in = torch.cuda.Event()
                self._map_ready, self._map_out = torch.cuda.Event(), torch.cuda.Event()
            self._half = self.half_detector()
        s = self.stream
        m, n = pages_h.shape[0], crops_h.shape[0]
        hb = self._half.input_shape[0] if self._half is not None else m
        halves = [(0, min(m, hb))] + ([(hb, m)] if m > hb else [])
        # Copies start after everything already queued on the pipeline's
        # stream (the previous batch's readers of the staging buffers).
        self._h2d.wait_stream(s)
        with torch.cuda.stream(self._h2d):
            for k, (a, b) in enumerate(halves):
                self._stage_pages[a:b].copy_(pages_h[a:b], non_blocking=True)
                self._half_in[k].record(self._h2d)
            self._stage_crops[:n].copy_(crops_h, non_blocking=True)
            self._crops_in.record(self._h2d)
        for k, (a, b) in enumerate(halves):
            s.wait_event(self._half_in[k])
            if self._half is not None:
                self._half.enqueue_nhwc(self._stage_pages[a:b], self.prob[a:], s)
            else:
                self.det.enqueue_nhwc(self._stage_pages[a:b], self.prob, s)
        px = m * self.size * self.size
        capi.check(self.lib.ppocr_b200_binarize(_p(self.prob), _p(self.bitmap), px, self.thresh,
                                                ctypes.c_void_p(s.cuda_stream)))
        self._map_ready.record(s)
        self._d2h.wait_event(self._map_ready)
        with torch.cuda.stream(self._d2h):
            bitmap_h.view(-1)[:px].copy_(self.bitmap.view(-1)[:px], non_blocking=True)
            self._map_out.record(self._d2h)
        s.wait_event(self._crops_in)
        self.rec.enqueue(self._stage_crops[:n])
        with torch.cuda.stream(s):
            ids_h[:n].copy_(self.rec.out_ids[:n], non_blocking=True)
            len_h[:n].copy_(self.rec.out_len[:n], non_blocking=True)
            score_h[:n].copy_(self.rec.out_score[:n], non_blocking=True)
        s.wait_event(self._map_out)

    def half_detector(self):
        """The compiled shape with half the detector's pages (same size and
        weights file), or None when the catalog has none."""
        half = self.pages // 2
        name = f"det_b{half}" if self.size == 960 else None
        if not half or name is None or name not in models.SHAPES:
            return None
        return CompiledModel(name, self.device)

    def close(self) -> None:
        self.det.close()
        self.rec.close()
        if getattr(self, "_half", None) is not None:
            self._half.close()
