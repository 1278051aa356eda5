"""Operator parity on the B200: every kernel through the C-ABI
(include/ppocr_b200_ops.h, include/ppocr_b200_head.h) against the CPU oracle
(oracle/layers.py, oracle/ctc_oracle.c) on the same seeded inputs."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import ptr, stream_handle
from helpers import assert_close, dev, f16, host, rng
from oracle import layers as L

pytestmark = pytest.mark.gpu


def sync():
    torch.cuda.synchronize()


def check_device_error(native):
    assert native.ppocr_b200_device_error() == 0, "a kernel's bounded wait ran out"


# ------------------------------------------------------------ tensor cores
GEMM_CASES = [
    # rows, ci, co, bias, residual, act
    (256, 128, 128, True, False, 1),
    (1000, 120, 360, True, False, 0),   # K tail (120), N tail (360), M tail
    (333, 240, 120, True, True, 0),     # residual epilogue
    (130, 64, 48, True, False, 1),      # N tile 48
    (2048, 1024, 1024, True, False, 1),
    (512, 2048, 120, True, False, 0),
    (77, 120, 240, True, False, 5),     # swish
    (300, 64, 128, True, False, 3),     # hardswish
    (1, 128, 64, False, False, 0),      # single row, no bias
    # 256-row tiles (K >= 32 k-blocks, >= 4 tiles per SM), partial last tile
    (40000, 2048, 1024, True, False, 1),
    (37900, 2048, 1024, True, True, 0),
    # 256-row tiles for short K at N <= 128 (double-buffered accumulator)
    (76000, 64, 128, True, False, 3),
    (80000, 120, 64, True, True, 0),
    # 128-row tiles drained by two warps per lane quarter, one column half
    # each (N tiles of 128 and 256), bias / residual fetched ahead
    (20480, 120, 120, True, True, 0),
    (10240, 120, 240, True, True, 5),
    (3000, 240, 256, False, True, 1),
    # N tile 64 at 128 rows: four of the eight epilogue warps drain it
    (1000, 64, 64, True, True, 1),
    # 256 x 128 tiles for short K (<= 8 k-blocks) at N >= 256
    (80000, 512, 512, True, False, 1),
]


@pytest.mark.parametrize("rows,ci,co,bias,residual,act", GEMM_CASES)
def test_gemm_epilogue(native, cuda, rows, ci, co, bias, residual, act):
    r = rng(rows + ci + co)
    x = f16(r.uniform(-1, 1, (rows, ci)))
    w = f16(r.standard_normal((co, ci)) * np.sqrt(2.0 / ci))
    b = f16(r.normal(0, 0.1, co)) if bias else None
    res = f16(r.uniform(-1, 1, (rows, co))) if residual else None
    y = torch.empty(rows, co, dtype=torch.float16, device=cuda)
    dx, dw = dev(x), dev(w)
    db = dev(b) if bias else None
    dr = dev(res) if residual else None
    rc = native.ppocr_b200_gemm_epilogue(ptr(dx), ptr(dw), ptr(db) if bias else None,
                                         ptr(dr) if residual else None, ptr(y), rows, ci, co, act,
                                         stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    want = L.gemm(x, w, b, res, act)
    assert_close(host(y), want, what=f"gemm {rows}x{ci}x{co}")


CONV_CASES = [
    # batch, h, w, ci, co, k
    (2, 3, 80, 64, 128, 3),
    (2, 6, 80, 128, 256, 3),
    (1, 24, 160, 48, 48, 3),    # Ci 48 (channel tail), N tile 48
    (2, 30, 30, 64, 64, 3),     # width not a multiple of 16
    (1, 12, 80, 48, 128, 3),
    (1, 7, 9, 64, 64, 5),       # 5x5, tiny image
    (3, 3, 80, 512, 256, 3),
    # 256-row tiles: whole-row boxes (OW 80: 3 rows per tile; OW 64: 4 rows,
    # partial last tile) and 32-pixel segments (OW 160)
    (316, 3, 80, 512, 512, 3),
    (301, 5, 64, 512, 512, 3),
    (160, 3, 160, 512, 512, 3),
    # 256-row tiles with double-buffered accumulators (N tile <= 128):
    (130, 7, 80, 64, 128, 3),   # N 128, partial last tile
    (40, 6, 80, 128, 512, 3),   # N 512 with a short K loop -> 128-column tiles
    (64, 12, 128, 64, 64, 3),   # N 64, 128-pixel rows
    (24, 24, 160, 48, 48, 3),   # N 48 (direct-store epilogue), rows in 2 parts of 80
    (10, 16, 480, 48, 48, 3),   # rows of 480 in 6 parts of 80
]


@pytest.mark.parametrize("batch,h,w,ci,co,k", CONV_CASES)
def test_implicit_conv(native, cuda, batch, h, w, ci, co, k):
    r = rng(batch * 7 + h + w + ci + co)
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    wt = f16(r.standard_normal((co, k, k, ci)) * np.sqrt(2.0 / (ci * k * k)))
    b = f16(r.normal(0, 0.1, co))
    y = torch.empty(batch, h, w, co, dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    p = k // 2
    rc = native.ppocr_b200_conv_nhwc(ptr(dx), ptr(dw), ptr(db), ptr(y), batch, ci, h, w, co, k, k,
                                     1, 1, p, p, 1, 1, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    want = L.conv_nhwc(x, wt, b, (1, 1), (p, p), 1, 1)
    assert_close(host(y), want, what=f"conv{k}x{k} {batch}x{h}x{w}x{ci}->{co}")


HALO_CASES = [
    # batch, h, w, ci, co, act: few-channel 3x3 convs staged as halo slabs
    (3, 11, 37, 16, 32, 2),     # Ci 16, N tile 48 for Co 32, runtime activation switch (GELU)
    (2, 5, 200, 32, 80, 0),     # Co 80 in a 128-wide tile, no activation, width in column blocks
    (1, 40, 33, 64, 112, 1),    # Ci 64, partial row blocks
    (5, 1, 300, 48, 48, 1),     # single-row images
]


@pytest.mark.parametrize("batch,h,w,ci,co,act", HALO_CASES)
def test_halo_conv(native, cuda, batch, h, w, ci, co, act):
    r = rng(500 + batch + h + w + ci + co)
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    wt = f16(r.standard_normal((co, 3, 3, ci)) * np.sqrt(2.0 / (ci * 9)))
    b = f16(r.normal(0, 0.1, co))
    y = torch.full((batch, h, w, co), float("nan"), dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    rc = native.ppocr_b200_conv_nhwc(ptr(dx), ptr(dw), ptr(db), ptr(y), batch, ci, h, w, co, 3, 3,
                                     1, 1, 1, 1, 1, act, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    want = L.conv_nhwc(x, wt, b, (1, 1), (1, 1), 1, act)
    assert_close(host(y), want, what=f"halo conv {batch}x{h}x{w}x{ci}->{co} act {act}")


DWPW_CASES = [
    # batch, h, w, k, co, act_dw, act_pw, bias
    (2, 48, 320, 5, 128, 3, 3, True),    # BASELINE config 2's block
    (3, 7, 100, 5, 128, 3, 3, True),     # odd height, width not a multiple of 64
    (2, 9, 30, 3, 64, 1, 1, True),       # 3x3, Co 64, ReLU
    (1, 5, 70, 5, 64, 2, 0, False),      # no biases (depthwise activation not applied), runtime switch
]


@pytest.mark.parametrize("batch,h,w,k,co,act_dw,act_pw,bias", DWPW_CASES)
def test_dwpw_block(native, cuda, batch, h, w, k, co, act_dw, act_pw, bias):
    """Fused depthwise + pointwise block against the oracle's two separate
    operators (depthwise in the reference's tap order, fp16-rounded
    intermediate, then the GEMM)."""
    r = rng(600 + h + w + k + co)
    x = f16(r.uniform(-1, 1, (batch, h, w, 64)))
    wd = f16(r.normal(0, 0.3, (64, k, k)))
    bd = f16(r.normal(0, 0.1, 64)) if bias else None
    wp = f16(r.standard_normal((co, 64)) * np.sqrt(2.0 / 64))
    bp = f16(r.normal(0, 0.1, co)) if bias else None
    y = torch.full((batch, h, w, co), float("nan"), dtype=torch.float16, device=cuda)
    dx, dwd, dwp = dev(x), dev(wd), dev(wp)
    dbd = dev(bd) if bias else None
    dbp = dev(bp) if bias else None
    rc = native.ppocr_b200_dwpw_block(ptr(dx), ptr(dwd), ptr(dbd) if bias else None, act_dw, ptr(dwp),
                                      ptr(dbp) if bias else None, act_pw, ptr(y), batch, h, w, 64, k, co,
                                      stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    mid = L.depthwise_exact(x, wd, bd if bias else torch.zeros(64), (1, 1), (k // 2, k // 2), act_dw if bias else 0)
    want = L.gemm(mid, wp, bp, None, act_pw)
    assert_close(host(y), want, what=f"dwpw {batch}x{h}x{w} k{k} -> {co}")


@pytest.mark.parametrize("batch,h,w,co,act", [(2, 48, 320, 48, 1), (1, 9, 35, 48, 1), (2, 10, 12, 32, 1),
                                             (1, 8, 8, 64, 0), (3, 50, 96, 16, 3), (2, 47, 64, 32, 1),
                                             (600, 48, 320, 48, 1), (4, 48, 320, 48, 0), (2, 32, 64, 64, 5)])
def test_stem_direct_conv(native, cuda, batch, h, w, co, act):
    """Stem 3x3 stride-2 conv with 3 input channels: the tensor-core form
    (rows a multiple of 16 bytes: odd heights, partial units, many images)
    and the SIMT form (odd output widths leave a single pixel in the last
    pair)."""
    r = rng(3 + w)
    x = f16(r.uniform(-1, 1, (batch, h, w, 3)))
    wt = f16(r.standard_normal((co, 3, 3, 3)) * np.sqrt(2.0 / 27))
    b = f16(r.normal(0, 0.1, co))
    oh, ow = (h + 2 - 3) // 2 + 1, (w + 2 - 3) // 2 + 1
    y = torch.empty(batch, oh, ow, co, dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    rc = native.ppocr_b200_conv_nhwc(ptr(dx), ptr(dw), ptr(db), ptr(y), batch, 3, h, w, co, 3, 3,
                                     2, 2, 1, 1, 1, act, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    want = L.conv_nhwc(x, wt, b, (2, 2), (1, 1), 1, act)
    assert_close(host(y), want, what=f"stem {batch}x{h}x{w} -> {co} act {act}")


@pytest.mark.parametrize("batch,h,w,ci,co,act", [(2, 48, 320, 3, 48, 1), (1, 9, 35, 3, 48, 1),
                                                 (3, 10, 12, 3, 32, 0), (1, 7, 8, 1, 64, 1),
                                                 (40, 48, 320, 3, 48, 1)])
def test_stem_space_to_depth(native, cuda, batch, h, w, ci, co, act):
    """Stem 3x3 stride-2 pad-1 conv on the tensor cores through the
    space-to-depth image (odd heights/widths leave zero sub-pixels; 40 lines
    are enough for 256-row tiles)."""
    r = rng(5 + w + ci)
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    wt = f16(r.standard_normal((co, 3, 3, ci)) * np.sqrt(2.0 / (9 * ci)))
    b = f16(r.normal(0, 0.1, co))
    oh, ow = (h + 1) // 2, (w + 1) // 2
    y = torch.empty(batch, oh, ow, co, dtype=torch.float16, device=cuda)
    wp = torch.empty(co * 64, dtype=torch.float16, device=cuda)
    nbytes = native.ppocr_b200_stem_s2d_scratch_bytes(batch, h, w)
    assert nbytes == batch * oh * ow * 32
    scratch = torch.empty(nbytes // 2, dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    assert native.ppocr_b200_stem_s2d_pack(ptr(dw), ptr(wp), co, ci, stream_handle()) == 0
    rc = native.ppocr_b200_stem_conv_s2d(ptr(dx), ptr(wp), ptr(db), ptr(y), ptr(scratch), batch, ci, h, w, co,
                                         act, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    want = L.conv_nhwc(x, wt, b, (2, 2), (1, 1), 1, act)
    assert_close(host(y), want, what=f"stem s2d {batch}x{h}x{w}x{ci}->{co}")


# ------------------------------------------------------------ depthwise
DW_CASES = [
    # batch, h, w, c, kh, kw, sh, sw, act
    (2, 24, 160, 48, 3, 3, 2, 2, 1),
    (2, 12, 80, 128, 3, 3, 2, 1, 1),
    (2, 3, 80, 1024, 3, 3, 1, 1, 1),
    (2, 48, 320, 64, 5, 5, 1, 1, 3),   # BASELINE config 2 depthwise 5x5
    (1, 9, 33, 16, 1, 7, 1, 1, 0),
    (1, 20, 20, 8, 9, 9, 1, 1, 2),
]


@pytest.mark.parametrize("batch,h,w,c,kh,kw,sh,sw,act", DW_CASES)
def test_depthwise_bit_exact(native, cuda, batch, h, w, c, kh, kw, sh, sw, act):
    """Same fp32 FMA tap order as the reference kernel, so bit-exact."""
    r = rng(h * w + c + kh)
    x = f16(r.uniform(-1, 1, (batch, h, w, c)))
    wt = f16(r.standard_normal((c, kh, kw)) * np.sqrt(2.0 / (kh * kw)))
    b = f16(r.normal(0, 0.1, c))
    ph, pw = kh // 2, kw // 2
    oh, ow = (h + 2 * ph - kh) // sh + 1, (w + 2 * pw - kw) // sw + 1
    y = torch.empty(batch, oh, ow, c, dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    rc = native.ppocr_b200_conv_nhwc(ptr(dx), ptr(dw), ptr(db), ptr(y), batch, c, h, w, c, kh, kw,
                                     sh, sw, ph, pw, c, act, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    want = L.depthwise_exact(x, wt, b, (sh, sw), (ph, pw), act)
    got = host(y)
    if act in (0, 1, 3):
        assert torch.equal(got, want), f"max diff {(got - want).abs().max().item()}"
    else:
        assert_close(got, want, what="depthwise gelu")


# ------------------------------------------------------------ sequence ops
@pytest.mark.parametrize("rows,cols", [(10240, 120), (77, 120), (33, 40), (129, 64), (50, 200), (9, 256),
                                       (31, 100), (5, 24)])
def test_layernorm(native, cuda, rows, cols):
    """Vectorised lane-group form (cols a multiple of 8 in (32, 256], ragged
    row counts) and the scalar form (other widths)."""
    r = rng(11 + cols)
    x = f16(r.standard_normal((rows, cols)) * 2 + 0.5)
    s = f16(r.normal(1, 0.1, cols))
    b = f16(r.normal(0, 0.1, cols))
    y = torch.empty(rows, cols, dtype=torch.float16, device=cuda)
    dx, ds, dbb = dev(x), dev(s), dev(b)
    assert native.ppocr_b200_layernorm(ptr(dx), ptr(ds), ptr(dbb), ptr(y), rows, cols, 1e-6,
                                       stream_handle()) == 0
    sync()
    assert_close(host(y), L.layernorm(x, s, b, 1e-6), what="layernorm")


def test_softmax(native, cuda):
    r = rng(12)
    x = f16(r.standard_normal((4096, 40)) * 3)
    y = torch.empty(4096, 40, dtype=torch.float16, device=cuda)
    dx = dev(x)
    assert native.ppocr_b200_softmax(ptr(dx), ptr(y), 4096, 40, stream_handle()) == 0
    sync()
    assert_close(host(y), L.softmax(x), what="softmax")


@pytest.mark.parametrize("batches,m,n,k", [(16, 40, 40, 15), (16, 40, 15, 40), (3, 200, 300, 130), (1, 5, 7, 3),
                                           (2, 129, 17, 64), (4, 33, 64, 65), (2, 16, 128, 0),
                                           # more batches than one grid's z extent: two launches
                                           (70000, 2, 3, 5)])
def test_matmul_batched(native, cuda, batches, m, n, k):
    """Runtime::matmul with a computed right-hand side (the exporter's
    attention products; tensor cores with SIMT-staged operands): fp32
    accumulation, one fp16 rounding, against the oracle; k = 0 gives zeros."""
    r = rng(30 + m + n + k)
    a = f16(r.standard_normal((batches, m, k)))
    b = f16(r.standard_normal((batches, k, n)))
    y = torch.full((batches, m, n), 7.0, dtype=torch.float16, device=cuda)
    assert native.ppocr_b200_matmul(ptr(dev(a)), ptr(dev(b)), ptr(y), batches, m, n, k, stream_handle()) == 0
    sync()
    check_device_error(native)
    assert_close(host(y), L.matmul(a, b), what="matmul")


@pytest.mark.parametrize("lines,seq,heads,dh", [(4, 40, 8, 15), (3, 25, 4, 16), (2, 20, 2, 24), (2, 70, 2, 8),
                                               (1, 10, 2, 40), (3, 17, 3, 5), (2, 64, 8, 16),
                                               (5, 40, 3, 7), (2, 40, 12, 16), (600, 40, 8, 15),
                                               # tensor-core path edges: one line (a group of three with
                                               # two empty), one head, head_dim 1, odd head widths
                                               (1, 40, 1, 1), (7, 40, 16, 4), (3, 40, 5, 9)])
def test_attention(native, cuda, lines, seq, heads, dh):
    r = rng(13 + seq)
    qkv = f16(r.standard_normal((lines, seq, 3 * heads * dh)))
    y = torch.empty(lines, seq, heads * dh, dtype=torch.float16, device=cuda)
    d = dev(qkv)
    scale = float(np.float32(dh ** -0.5))
    assert native.ppocr_b200_attention(ptr(d), ptr(y), lines, seq, heads, dh, scale, stream_handle()) == 0
    sync()
    assert_close(host(y), L.attention(qkv, heads, dh, scale), what="attention")


def test_pools(native, cuda):
    r = rng(14)
    x = f16(r.uniform(-2, 2, (3, 3, 80, 256)))
    y = torch.empty(3, 1, 40, 256, dtype=torch.float16, device=cuda)
    d = dev(x)
    assert native.ppocr_b200_pool_nhwc(ptr(d), ptr(y), 3, 256, 3, 80, 3, 2, 3, 2, 0, 0, 0, stream_handle()) == 0
    sync()
    assert_close(host(y), L.pool_nhwc(x, (3, 2), (3, 2), (0, 0), False), what="avgpool")
    y2 = torch.empty(3, 2, 79, 256, dtype=torch.float16, device=cuda)
    assert native.ppocr_b200_pool_nhwc(ptr(d), ptr(y2), 3, 256, 3, 80, 2, 2, 1, 1, 0, 0, 1, stream_handle()) == 0
    sync()
    assert torch.equal(host(y2), L.pool_nhwc(x, (2, 2), (1, 1), (0, 0), True))


@pytest.mark.parametrize("b,c,h,w,oh,ow", [(1, 24, 13, 7, 32, 20), (3, 16, 5, 5, 40, 35), (2, 8, 9, 9, 9, 9)])
def test_resize_nearest_shapes(native, cuda, b, c, h, w, oh, ow):
    """Non-integer and identity scales through the 16-byte-group form."""
    r = rng(80 + oh)
    x = f16(r.uniform(-1, 1, (b, h, w, c)))
    y = torch.empty(b, oh, ow, c, dtype=torch.float16, device=cuda)
    sh, sw = float(np.float32(oh) / np.float32(h)), float(np.float32(ow) / np.float32(w))
    dx = dev(x)
    assert native.ppocr_b200_resize_nearest_nhwc(ptr(dx), None, ptr(y), b, c, h, w, oh, ow, sh, sw,
                                                 stream_handle()) == 0
    sync()
    assert torch.equal(host(y), L.resize_nearest_nhwc(x, oh, ow, sh, sw))


def test_resize_add_and_concat(native, cuda):
    r = rng(15)
    x = f16(r.uniform(-1, 1, (2, 15, 15, 64)))
    a = f16(r.uniform(-1, 1, (2, 30, 30, 64)))
    y = torch.empty(2, 30, 30, 64, dtype=torch.float16, device=cuda)
    dx, da = dev(x), dev(a)
    assert native.ppocr_b200_resize_nearest_nhwc(ptr(dx), ptr(da), ptr(y), 2, 64, 15, 15, 30, 30, 2.0, 2.0,
                                                 stream_handle()) == 0
    sync()
    assert torch.equal(host(y), L.resize_nearest_nhwc(x, 30, 30, 2.0, 2.0, addend=a))
    c = torch.empty(2 * 30 * 30, 128, dtype=torch.float16, device=cuda)
    assert native.ppocr_b200_concat(ptr(da), ptr(y), ptr(c), 2 * 30 * 30, 64, 64, stream_handle()) == 0
    sync()
    want = torch.cat([a.reshape(-1, 64), L.resize_nearest_nhwc(x, 30, 30, 2.0, 2.0, addend=a).reshape(-1, 64)], 1)
    assert torch.equal(host(c), want)


@pytest.mark.parametrize("batch,oh,ow,levels", [
    (2, 48, 40, [(64, 1), (64, 2), (64, 4), (64, 8)]),   # the DB FPN tail: four levels, factors 1..8
    (1, 30, 30, [(16, 1), (8, 3), (32, 2)]),             # mixed channel counts, a factor of 3
    (3, 17, 11, [(8, 1)]),                               # one source: a plain copy
])
def test_upsample_concat(native, cuda, batch, oh, ow, levels):
    """The fused FPN tail equals the chain of nearest resizes + concats bit
    for bit (same index mapping, pure copies)."""
    r = rng(70 + oh)
    xs = [f16(r.uniform(-1, 1, (batch, oh // f, ow // f, c))) for c, f in levels]
    ds = [dev(x) for x in xs]
    ctot = sum(c for c, _ in levels)
    y = torch.full((batch, oh, ow, ctot), float("nan"), dtype=torch.float16, device=cuda)
    n = len(levels)
    srcs = (ctypes.c_void_p * n)(*[d.data_ptr() for d in ds])
    chans = (ctypes.c_int * n)(*[c for c, _ in levels])
    hs = (ctypes.c_int * n)(*[x.shape[1] for x in xs])
    ws = (ctypes.c_int * n)(*[x.shape[2] for x in xs])
    assert native.ppocr_b200_upsample_concat_nhwc(srcs, chans, hs, ws, n, ptr(y), batch, oh, ow,
                                                  stream_handle()) == 0, native.ppocr_b200_last_error()
    sync()
    want = torch.cat([L.resize_nearest_nhwc(x, oh, ow, np.float32(oh) / np.float32(x.shape[1]),
                                            np.float32(ow) / np.float32(x.shape[2])) for x in xs], -1)
    assert torch.equal(host(y), want)


STREAM_CASES = [
    # batch, h, w, ci, co, act: wide-input 3x3 convs with Co <= 64, staged
    # per filter row and 64-channel chunk with the filter streamed; the slab
    # plan (rows x columns, tiles per slab, ring depth) follows from the
    # shape and the SM count
    (1, 240, 240, 256, 64, 1),  # the C5 FPN / DB-head layer: 2-row slabs, 4 tiles, 2-deep ring
    (8, 60, 60, 256, 64, 0),    # C5's 60^2 level: 4-row slabs, 2 tiles, 3-deep ring, no activation
    (8, 30, 30, 256, 64, 1),    # C5's 30^2 level: 4-row one-tile slabs, 4-deep ring, partial row block
    (4, 96, 96, 256, 64, 1),    # 3 tiles per slab, 3 column blocks of 32
    (2, 32, 32, 128, 64, 1),    # Ci 128 (2 chunks), 2 column blocks
    (1, 7, 100, 256, 32, 2),    # Co 32 (filter rows past Co zero-filled), single-row slabs, GELU switch
    (3, 5, 254, 512, 48, 1),    # 8 chunks, Co 48, many narrow column blocks
    (1, 9, 300, 192, 64, 1),    # 3 chunks, width in column blocks
    (2, 4, 4, 256, 64, 1),      # tiny images: one tile, most rows discarded
]


@pytest.mark.parametrize("batch,h,w,ci,co,act", STREAM_CASES)
def test_halo_stream_conv(native, cuda, batch, h, w, ci, co, act):
    r = rng(700 + batch + h + w + ci + co)
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    wt = f16(r.standard_normal((co, 3, 3, ci)) * np.sqrt(2.0 / (ci * 9)))
    b = f16(r.normal(0, 0.1, co))
    y = torch.full((batch, h, w, co), float("nan"), dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    rc = native.ppocr_b200_conv_nhwc(ptr(dx), ptr(dw), ptr(db), ptr(y), batch, ci, h, w, co, 3, 3,
                                     1, 1, 1, 1, 1, act, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    want = L.conv_nhwc(x, wt, b, (1, 1), (1, 1), 1, act)
    assert_close(host(y), want, what=f"streamed halo conv {batch}x{h}x{w}x{ci}->{co} act {act}")


DECONV_CASES = [
    # batch, h, w, ci, co, act, bias
    (2, 16, 16, 64, 64, 1, True),     # tensor-core path (Co % 64 == 0)
    (2, 16, 16, 64, 1, 4, True),      # one output channel: SIMT path, sigmoid
    (1, 7, 30, 64, 128, 0, True),     # tensor cores, ragged 16-pixel segments
    (2, 12, 64, 64, 64, 1, False),    # tensor cores, 32-pixel segments, no bias
    (1, 9, 11, 24, 3, 0, True),       # 12 outputs per pixel, Ci not a multiple of 8
    (1, 5, 7, 128, 1, 4, False),      # 16 threads per input pixel, partial warp at the end
    (3, 33, 29, 64, 1, 4, True),      # 8 threads per pixel, grid-stride with a ragged tail
    (1, 6, 10, 256, 1, 4, True),      # 32 threads per pixel (a whole warp per input pixel)
    (3, 240, 240, 64, 1, 4, True),    # more pixels than the capped grid covers in one pass
]


@pytest.mark.parametrize("batch,h,w,ci,co,act,bias", DECONV_CASES)
def test_deconv(native, cuda, batch, h, w, ci, co, act, bias):
    r = rng(16 + co + h)
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    wt = f16(r.standard_normal((ci, 2, 2, co)) * np.sqrt(2.0 / (4 * ci)))
    b = f16(r.normal(0, 0.1, co)) if bias else None
    y = torch.empty(batch, 2 * h, 2 * w, co, dtype=torch.float16, device=cuda)
    dx, dw = dev(x), dev(wt)
    db = dev(b) if bias else None
    assert native.ppocr_b200_deconv_nhwc(ptr(dx), ptr(dw), ptr(db) if bias else None, ptr(y), batch, h, w, ci,
                                         co, 2, 2, act, stream_handle()) == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    assert_close(host(y), L.deconv_kxk(x, wt, b, act), what=f"deconv {batch}x{h}x{w}x{ci}->{co}")


DB_TAIL_CASES = [
    # batch, h, w, ci, act, act2, bias: the DB head's two transposed convs
    # (ci -> 64 -> 1, 2x2 stride 2) fused, against the two separate ops
    (1, 240, 240, 64, 1, 4, True),    # the C5 head at one page: 256-row x 128-column tiles
    (2, 32, 32, 64, 1, 4, True),      # few tiles: 128-row x 256-column tiles, column-split epilogue
    (3, 17, 50, 64, 1, 4, False),     # ragged 16-pixel segments (width 50), no biases
    (1, 9, 64, 128, 0, 0, True),      # Ci 128 (two k-blocks), no activations, 32-pixel segments
    (2, 6, 10, 64, 2, 4, True),       # runtime activation switch (GELU) in the first conv
]


@pytest.mark.parametrize("batch,h,w,ci,act,act2,bias", DB_TAIL_CASES)
def test_deconv_db_tail(native, cuda, batch, h, w, ci, act, act2, bias):
    """Fused DB tail bit-identical to deconv(ci -> 64) then deconv(64 -> 1),
    and within the fp16 bar of the oracle."""
    r = rng(80 + h + w + ci)
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    w1 = f16(r.standard_normal((ci, 2, 2, 64)) * np.sqrt(2.0 / (4 * ci)))
    b1 = f16(r.normal(0, 0.1, 64)) if bias else None
    w2 = f16(r.standard_normal((64, 2, 2, 1)) * np.sqrt(2.0 / 256))
    b2 = f16(r.normal(0, 0.1, 1)) if bias else None
    dx, dw1, dw2 = dev(x), dev(w1), dev(w2)
    db1, db2 = (dev(b1), dev(b2)) if bias else (None, None)
    mid = torch.empty(batch, 2 * h, 2 * w, 64, dtype=torch.float16, device=cuda)
    want = torch.full((batch, 4 * h, 4 * w, 1), float("nan"), dtype=torch.float16, device=cuda)
    got = torch.full((batch, 4 * h, 4 * w, 1), float("nan"), dtype=torch.float16, device=cuda)
    s = stream_handle()
    assert native.ppocr_b200_deconv_nhwc(ptr(dx), ptr(dw1), ptr(db1) if bias else None, ptr(mid), batch, h, w, ci,
                                         64, 2, 2, act, s) == 0, native.ppocr_b200_last_error()
    assert native.ppocr_b200_deconv_nhwc(ptr(mid), ptr(dw2), ptr(db2) if bias else None, ptr(want), batch,
                                         2 * h, 2 * w, 64, 1, 2, 2, act2, s) == 0, native.ppocr_b200_last_error()
    for _ in range(2):  # twice: the same bits on a repeat
        assert native.ppocr_b200_deconv_db_tail(ptr(dx), ptr(dw1), ptr(db1) if bias else None, act, ptr(dw2),
                                                ptr(db2) if bias else None, act2, ptr(got), batch, h, w, ci,
                                                s) == 0, native.ppocr_b200_last_error()
        sync()
        check_device_error(native)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    ref = L.deconv_kxk(L.deconv_kxk(x, w1, b1, act), w2, b2, act2)
    assert_close(host(got), ref, what=f"db tail {batch}x{h}x{w}x{ci}")


@pytest.mark.parametrize("kh,kw,ci", [(1, 2, 64), (2, 1, 128), (1, 1, 64)])
def test_deconv_fewer_taps(native, cuda, kh, kw, ci):
    """Kernel == stride with fewer than four outputs per input pixel: the
    grouped kernel's lanes that own no output store nothing."""
    r = rng(40 + kh * 3 + kw)
    batch, h, w, co = 2, 9, 13, 1
    x = f16(r.uniform(-1, 1, (batch, h, w, ci)))
    wt = f16(r.standard_normal((ci, kh, kw, co)) * np.sqrt(2.0 / (kh * kw * ci)))
    b = f16(r.normal(0, 0.1, co))
    y = torch.full((batch, kh * h, kw * w, co), float("nan"), dtype=torch.float16, device=cuda)
    dx, dw, db = dev(x), dev(wt), dev(b)
    assert native.ppocr_b200_deconv_nhwc(ptr(dx), ptr(dw), ptr(db), ptr(y), batch, h, w, ci, co, kh, kw, 4,
                                         stream_handle()) == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    assert_close(host(y), L.deconv_kxk(x, wt, b, 4), what=f"deconv {kh}x{kw} {ci}->1")


@pytest.mark.parametrize("n", [960 * 960 + 3, 5, 3, 1, 4096 * 4 + 7])
def test_binarize_bit_exact(native, cuda, n):
    r = rng(17)
    p = r.uniform(0, 1, n).astype(np.float32)
    edge = [0.3, np.nextafter(np.float32(0.3), 1), np.nextafter(np.float32(0.3), 0), 0.0, 1.0]
    p[:min(5, n)] = edge[:min(5, n)]
    d = torch.from_numpy(p).cuda()
    m = torch.empty(p.size, dtype=torch.uint8, device=cuda)
    assert native.ppocr_b200_binarize(ptr(d), ptr(m), p.size, 0.3, stream_handle()) == 0
    sync()
    assert np.array_equal(m.cpu().numpy(), L.binarize(p, 0.3))


# ------------------------------------------------------------ CTC head
def test_logits_argmax_and_collapse(native, cuda, oracle_c):
    """BASELINE config 1 at its full size: [32, 40, 18385] FP16 logits."""
    from ppocr_b200 import workloads

    r = rng(18)
    lines, T, V = 32, 40, 18385
    logits = workloads.c1_logits(r, lines, T, V)
    rows = lines * T
    d = torch.from_numpy(logits.reshape(rows, V)).cuda()
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    prob = torch.empty(rows, dtype=torch.float32, device=cuda)
    mx = torch.empty(rows, dtype=torch.float32, device=cuda)
    assert native.ppocr_b200_logits_argmax_prob(ptr(d), rows, V, ptr(ids), ptr(prob), ptr(mx), 1,
                                                stream_handle()) == 0
    oid = torch.empty(lines, T, dtype=torch.int32, device=cuda)
    olen = torch.empty(lines, dtype=torch.int32, device=cuda)
    osc = torch.empty(lines, dtype=torch.float32, device=cuda)
    assert native.ppocr_b200_ctc_collapse(ptr(ids), ptr(prob), lines, T, 0, ptr(oid), ptr(olen), ptr(osc),
                                          stream_handle()) == 0
    sync()
    want_ids = np.empty(rows, np.int32)
    want_prob = np.empty(rows, np.float32)
    want_max = np.empty(rows, np.float32)
    oracle_c.oracle_argmax_prob(logits.ctypes.data, rows, V, want_ids.ctypes.data, want_prob.ctypes.data,
                                want_max.ctypes.data, 4)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(mx.cpu().numpy(), want_max)
    assert np.abs(prob.cpu().numpy() - want_prob).max() <= 1e-5
    # Collapse of the oracle's own ids/probs must match the device collapse
    # of the device ids/probs bit for bit on ids and lengths.
    c_ids = np.empty((lines, T), np.int32)
    c_len = np.empty(lines, np.int32)
    c_sc = np.empty(lines, np.float32)
    oracle_c.oracle_ctc_collapse(want_ids.ctypes.data, want_prob.ctypes.data, lines, T, 0, c_ids.ctypes.data,
                                 c_len.ctypes.data, c_sc.ctypes.data)
    assert np.array_equal(oid.cpu().numpy(), c_ids)
    assert np.array_equal(olen.cpu().numpy(), c_len)
    assert np.abs(osc.cpu().numpy() - c_sc).max() <= 1e-5


@pytest.mark.parametrize("rows,V,offset", [(3, 5, 0), (7, 1, 0), (64, 300, 0), (64, 300, 1),
                                           (40, 18385, 1), (33, 4099, 0), (6, 40001, 0), (5, 40001, 3),
                                           (9, 4088, 1), (5, 8185, 3), (7, 18424, 1), (4, 20473, 0),
                                           (3, 32760, 5), (3, 32761, 0), (300, 18385, 1), (445, 9001, 3),
                                           (1000, 18432, 0), (297, 8185, 5), (296, 18433, 0)])
def test_logits_argmax_shapes(native, cuda, oracle_c, rows, V, offset):
    """Edge cases: rows shorter than one 16-byte vector, odd vocabularies
    (rows start at any 2-byte offset), base pointers that are not 16-byte
    aligned, ties (repeated maxima), vocabularies at both sides of each
    register-resident row form's capacity, vocabularies past the largest
    one (the looping register form), and enough rows for the streaming form
    (one CTA per SM, two rows in flight) at both sides of its capacity."""
    r = rng(30 + V + offset)
    logits = r.standard_normal((rows, V)).astype(np.float16)
    logits[::3, V // 2] = 8.0
    logits[::3, V - 1] = 8.0  # tie: the lower id must win
    buf = torch.zeros(rows * V + offset, dtype=torch.float16, device=cuda)
    d = buf[offset:]
    d.copy_(torch.from_numpy(logits.reshape(-1)))
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    prob = torch.empty(rows, dtype=torch.float32, device=cuda)
    mx = torch.empty(rows, dtype=torch.float32, device=cuda)
    assert native.ppocr_b200_logits_argmax_prob(ptr(d), rows, V, ptr(ids), ptr(prob), ptr(mx), 1,
                                                stream_handle()) == 0
    sync()
    check_device_error(native)
    want_ids = np.empty(rows, np.int32)
    want_prob = np.empty(rows, np.float32)
    want_max = np.empty(rows, np.float32)
    oracle_c.oracle_argmax_prob(logits.ctypes.data, rows, V, want_ids.ctypes.data, want_prob.ctypes.data,
                                want_max.ctypes.data, 4)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(mx.cpu().numpy(), want_max)
    assert np.abs(prob.cpu().numpy() - want_prob).max() <= 1e-5


def test_collapse_bit_exact_on_device_inputs(native, cuda, oracle_c):
    """Same ids/probs in: lengths, ids and float scores identical."""
    r = rng(19)
    lines, T = 777, 40
    ids = r.integers(0, 6, (lines, T)).astype(np.int32)
    probs = r.random((lines, T)).astype(np.float32)
    d_ids, d_p = torch.from_numpy(ids).cuda(), torch.from_numpy(probs).cuda()
    oid = torch.empty(lines, T, dtype=torch.int32, device=cuda)
    olen = torch.empty(lines, dtype=torch.int32, device=cuda)
    osc = torch.empty(lines, dtype=torch.float32, device=cuda)
    assert native.ppocr_b200_ctc_collapse(ptr(d_ids), ptr(d_p), lines, T, 0, ptr(oid), ptr(olen), ptr(osc),
                                          stream_handle()) == 0
    sync()
    c_ids = np.empty((lines, T), np.int32)
    c_len = np.empty(lines, np.int32)
    c_sc = np.empty(lines, np.float32)
    oracle_c.oracle_ctc_collapse(ids.ctypes.data, probs.ctypes.data, lines, T, 0, c_ids.ctypes.data,
                                 c_len.ctypes.data, c_sc.ctypes.data)
    assert np.array_equal(oid.cpu().numpy(), c_ids)
    assert np.array_equal(olen.cpu().numpy(), c_len)
    assert np.array_equal(osc.cpu().numpy(), c_sc)


def _classifier_case(rows, H, V):
    r = rng(20 + V + H)
    hid = f16(r.standard_normal((rows, H)))
    w = f16(r.uniform(-1, 1, (H, V)) * np.sqrt(6.0 / (H + V)) * 4)
    b = f16(r.normal(0, 0.1, V))
    return hid, w, b


def _check_classifier(hid, w, b, ids, prob, mx):
    logits = hid.double() @ w.double() + b.double()
    top2 = torch.topk(logits, 2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 1e-3
    want_ids = logits.argmax(1)
    got_ids = ids.cpu().long()
    assert clear.float().mean() > 0.9
    assert torch.equal(got_ids[clear], want_ids[clear])
    want_prob = 1.0 / torch.exp(logits - logits.max(1, keepdim=True).values).sum(1)
    assert (prob.cpu().double() - want_prob).abs().max().item() <= 1e-4
    assert (mx.cpu().double() - logits.max(1).values).abs().max().item() <= 1e-3


@pytest.mark.parametrize("rows,H,V,tile", [(300, 128, 5000, 512), (1280, 128, 18385, 512),
                                           (1280, 128, 18385, 128), (77, 64, 2200, 64)])
def test_classifier_reference_signature(native, cuda, rows, H, V, tile):
    """Reference-signature entry (weight [H][V] as the worker holds it), with
    partial buffers sized by the reference's workspace shape: smaller than the
    B200 kernel's 256-column tiles need at tile 512 (the stream workspace is
    used), large enough at tiles 128 and 64 (the caller's buffers are)."""
    hid, w, b = _classifier_case(rows, H, V)
    dh, dw, db = dev(hid), dev(w), dev(b)
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    prob = torch.empty(rows, dtype=torch.float32, device=cuda)
    mx = torch.empty(rows, dtype=torch.float32, device=cuda)
    nrb, nvb, cnt = ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    assert native.ppocr_b200_classifier_workspace(rows, V, 16, tile, ctypes.byref(nrb), ctypes.byref(nvb),
                                                  ctypes.byref(cnt)) == 0
    pid = torch.empty(cnt.value, dtype=torch.int32, device=cuda)
    pmax = torch.empty(cnt.value, dtype=torch.float32, device=cuda)
    psum = torch.empty(cnt.value, dtype=torch.float32, device=cuda)
    rc = native.ppocr_b200_linear_argmax_prob(ptr(dh), ptr(dw), ptr(db), ptr(ids), ptr(prob), ptr(mx), rows, H, V,
                                              tile, ptr(pid), ptr(pmax), ptr(psum), 1, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    _check_classifier(hid, w, b, ids, prob, mx)
    # The reference rejects hidden sizes that are not multiples of 16.
    assert native.ppocr_b200_linear_argmax_prob(ptr(dh), ptr(dw), ptr(db), ptr(ids), ptr(prob), ptr(mx), rows, 120,
                                                V, 512, ptr(pid), ptr(pmax), ptr(psum), 1, stream_handle()) == -1


@pytest.mark.parametrize("rows,H,V", [(20480, 120, 18385), (16, 120, 300), (129, 64, 257),
                                      # vocabulary tile counts 8, 9, 11 (the four-threads-per-row merge,
                                      # uneven tile strides) with row counts off the 64-row block
                                      (1, 64, 2048), (65, 120, 2200), (130, 64, 2816)])
def test_classifier_packed(native, cuda, rows, H, V):
    """Packed-weight entry used by the pipeline (hidden 120, BASELINE)."""
    hid, w, b = _classifier_case(rows, H, V)
    dh, dw, db = dev(hid), dev(w), dev(b)
    packed = torch.empty(V, H, dtype=torch.float16, device=cuda)
    assert native.ppocr_b200_classifier_pack(ptr(dw), ptr(packed), H, V, stream_handle()) == 0
    tiles = (V + 255) // 256
    pid = torch.empty(rows * tiles, dtype=torch.int32, device=cuda)
    pmax = torch.empty(rows * tiles, dtype=torch.float32, device=cuda)
    psum = torch.empty(rows * tiles, dtype=torch.float32, device=cuda)
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    prob = torch.empty(rows, dtype=torch.float32, device=cuda)
    mx = torch.empty(rows, dtype=torch.float32, device=cuda)
    rc = native.ppocr_b200_classifier_run_packed(ptr(dh), ptr(packed), ptr(db), ptr(ids), ptr(prob), ptr(mx), rows,
                                                 H, V, ptr(pid), ptr(pmax), ptr(psum), 1, stream_handle())
    assert rc == 0, native.ppocr_b200_last_error()
    sync()
    check_device_error(native)
    _check_classifier(hid, w, b, ids, prob, mx)
