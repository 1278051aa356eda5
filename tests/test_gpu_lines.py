"""Line-tensor construction on the B200 against the oracle (the server's
write_line_tensor restated in numpy; the oracle is pinned to the server's own
unit tests in test_cpu_lines.py). Bar: f32 NCHW bit-exact, FP16 NHWC equal
to its round-to-nearest; over-wide lines fail with the reference's message."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import ptr, stream_handle
from helpers import rng
from oracle import lines as OL

pytestmark = pytest.mark.gpu
F32, F16 = 0, 1


def pack(images, pad=0):
    offs, buf, strides = [], [], []
    pos = 0
    for im in images:
        h, w = im.shape[:2]
        stride = w * 3 + pad
        rows = np.zeros((h, stride), np.uint8)
        rows[:, : w * 3] = im.reshape(h, -1)
        offs.append(pos)
        strides.append(stride)
        buf.append(rows.reshape(-1))
        pos += rows.size
    return np.concatenate(buf), offs, strides


def call(native, images, bucket, fmt, pad=0):
    data, offs, strides = pack(images, pad)
    n = len(images)
    d = torch.from_numpy(data).cuda()
    ws = [im.shape[1] for im in images]
    hs = [im.shape[0] for im in images]
    if fmt == F16:
        out = torch.full((n, 48, bucket, 3), float("nan"), dtype=torch.float16, device="cuda")
    else:
        out = torch.full((n, 3, 48, bucket), float("nan"), dtype=torch.float32, device="cuda")
    L = ctypes.c_longlong * n
    I = ctypes.c_int * n
    rc = native.ppocr_b200_line_tensors(ptr(d), L(*offs), I(*ws), I(*hs), I(*strides), n, bucket, ptr(out), fmt,
                                        stream_handle())
    torch.cuda.synchronize()
    return rc, out


def random_lines(r, n, bucket):
    ims = []
    for k in range(n):
        h = int(r.integers(8, 130))
        if k % 7 == 0:
            h = 48  # some lines already at the target height
        max_w = bucket * h // 48
        w = int(r.integers(1, max(2, max_w + 1)))
        if k % 7 == 0:
            w = min(w, bucket)  # h == 48: natural width == w -> copied
        ims.append(r.integers(0, 256, (h, w, 3), dtype=np.uint8))
    return ims


@pytest.mark.parametrize("n,bucket,pad", [(40, 320, 0), (9, 128, 5), (600, 320, 3)])
def test_line_tensors_match_oracle(native, cuda, n, bucket, pad):
    ims = random_lines(rng(800 + n + bucket), n, bucket)
    rc, got = call(native, ims, bucket, F32, pad)
    assert rc == 0, native.ppocr_b200_last_error()
    want = np.stack([OL.line_tensor(im, bucket) for im in ims])
    assert np.array_equal(got.cpu().numpy(), want)
    rc, got16 = call(native, ims, bucket, F16, pad)
    assert rc == 0, native.ppocr_b200_last_error()
    assert torch.equal(got16.cpu(), torch.from_numpy(want).permute(0, 2, 3, 1).half())


def test_line_tensors_golden_case_and_overflow(native, cuda):
    image = np.zeros((48, 129, 3), np.uint8)
    image[...] = [0, 127, 255]
    rc, got = call(native, [image], 640, F32)
    assert rc == 0
    t = got.cpu().numpy().reshape(-1)
    assert t[0] == -1.0 and t[2 * 48 * 640] == 1.0 and t[128] == -1.0 and t[129] == 0.0
    rc, _ = call(native, [image], 128, F32)
    assert rc == -1
    assert native.ppocr_b200_last_error() == b"line normalized width 129 exceeds maximum 128; split the line crop"
