"""The allocation-free classifier entry point
(ppocr_b200_classifier_run_packed_noalloc) against the regular packed entry
point, through the C-ABI, on two calls in a row.

It exists for callers that cannot call cudaMalloc on their serving path (for
example when all device memory belongs to the host's own pool allocator):
its scratch lives in a static device array of the library. This file is
collected last so that a run that stops at the first failure has already run
every other test; it also passes when run alone in a fresh process."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import ptr, stream_handle
from helpers import dev, f16, rng

pytestmark = pytest.mark.gpu


def _case(rows, H, V, seed):
    r = rng(900 + seed)
    hid = f16(r.standard_normal((rows, H)))
    w = f16(r.uniform(-1, 1, (H, V)) * np.sqrt(6.0 / (H + V)) * 4)
    b = f16(r.normal(0, 0.1, V))
    return hid, w, b


def _outputs(n, cuda):
    return (torch.empty(n, dtype=torch.int32, device=cuda), torch.empty(n, dtype=torch.float32, device=cuda),
            torch.empty(n, dtype=torch.float32, device=cuda))


@pytest.mark.parametrize("rows,H,V", [(20480, 120, 18385), (77, 64, 300)])
def test_noalloc_matches_packed_twice(native, cuda, rows, H, V):
    packed_ref = None
    for call in range(2):
        hid, w, b = _case(rows, H, V, call)
        dh, dw, db = dev(hid), dev(w), dev(b)
        packed = torch.empty(V, H, dtype=torch.float16, device=cuda)
        assert native.ppocr_b200_classifier_pack(ptr(dw), ptr(packed), H, V, stream_handle()) == 0
        tiles = (V + 255) // 256
        pid = torch.empty(rows * tiles, dtype=torch.int32, device=cuda)
        pmax = torch.empty(rows * tiles, dtype=torch.float32, device=cuda)
        psum = torch.empty(rows * tiles, dtype=torch.float32, device=cuda)
        ids, prob, mx = _outputs(rows, cuda)
        assert native.ppocr_b200_classifier_run_packed(
            ptr(dh), ptr(packed), ptr(db), ptr(ids), ptr(prob), ptr(mx), rows, H, V, ptr(pid), ptr(pmax),
            ptr(psum), 1, stream_handle()) == 0, native.ppocr_b200_last_error()
        ids2, prob2, mx2 = _outputs(rows, cuda)
        rc = native.ppocr_b200_classifier_run_packed_noalloc(
            ptr(dh), ptr(packed), ptr(db), ptr(ids2), ptr(prob2), ptr(mx2), rows, H, V, 1, stream_handle())
        assert rc == 0, native.ppocr_b200_last_error()
        torch.cuda.synchronize()
        # Same kernels and reduction order: identical results.
        assert torch.equal(ids2, ids)
        assert torch.equal(mx2, mx)
        assert (prob2 - prob).abs().max().item() <= 1e-6
        # Reads (and clears) the allocation-free path's own timeout word too.
        assert native.ppocr_b200_device_error() == 0


def test_noalloc_timeout_word_is_reported_once(native, cuda):
    """A code in the allocation-free head's timeout word (stored the way a
    projection whose bounded wait ran out stores it) is reported once by
    ppocr_b200_device_error() and then cleared."""
    assert native.ppocr_b200_device_error() == 0
    assert native.ppocr_b200_test_store_error_code(1, 77) == 0, native.ppocr_b200_last_error()
    assert native.ppocr_b200_device_error() == 77
    assert native.ppocr_b200_device_error() == 0


def test_noalloc_rejects_oversize(native, cuda):
    rows, H, V = 40000, 64, 18385  # 40000 * 72 partials > 2**21
    ids, prob, mx = _outputs(1, cuda)
    x = torch.empty(16, dtype=torch.float16, device=cuda)
    rc = native.ppocr_b200_classifier_run_packed_noalloc(ptr(x), ptr(x), ptr(x), ptr(ids), ptr(prob), ptr(mx),
                                                         rows, H, V, 1, stream_handle())
    assert rc == -1
    assert b"exceeds the allocation-free scratch limit" in native.ppocr_b200_last_error()
