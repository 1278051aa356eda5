"""torch-CPU float32 restatement of the layer operators (test oracle only).

Tensors are float32 holding fp16-representable values; rh() marks every point
where the reference stores an fp16 tensor (its Scalar = half storage,
native/src/compiled/runtime.cuh:40-41). Activation layouts are NHWC, filters
OHWI, as the exporter lays them out (tools/compiled_models/export.py:593-600).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def rh(x: torch.Tensor) -> torch.Tensor:
    """Round to fp16 and back (one fp16 store)."""
    return x.to(torch.float16).to(torch.float32)


def act(x: torch.Tensor, code: int) -> torch.Tensor:
    """Activation codes of the fused epilogues.

    0 none, 1 ReLU, 2 erf-GELU (spatial_kernels.cuh:31-42), 3 hardswish as the
    exporter's HardSigmoid(1/6, 1/2)*x chain, 4 sigmoid 1/(1+exp(-x))
    (runtime.cuh:118), 5 x*sigmoid(x), 6 hardsigmoid.
    """
    if code == 0:
        return x
    if code == 1:
        return torch.clamp_min(x, 0.0)
    if code == 2:
        return (x * (torch.erf(x / 1.41421354) + 1.0)) * 0.5
    if code == 3:
        return x * _hardsigmoid(x)
    if code == 4:
        return 1.0 / (1.0 + torch.exp(-x))
    if code == 5:
        return x * (1.0 / (1.0 + torch.exp(-x)))
    if code == 6:
        return _hardsigmoid(x)
    raise ValueError(code)


def _hardsigmoid(x):
    """clamp(alpha*x + beta) with alpha = float32(1/6), beta = 0.5, the
    multiply-add rounded once (as nvcc contracts the exporter's expression
    `(alpha)*(x)+(beta)` into an FMA)."""
    alpha = float(np.float32(0.166666671634))
    return torch.clamp((alpha * x.double() + 0.5).float(), 0.0, 1.0)


def epilogue(acc, bias=None, residual=None, code=0):
    """round(act(round(acc) + bias)) [+ residual after a round]."""
    v = rh(acc)
    if bias is not None:
        v = v + bias
    if residual is not None:
        v = rh(v) + residual
    return rh(act(v, code))


def conv_nhwc(x, w_ohwi, bias, stride, pad, groups, code):
    """Runtime::conv (runtime.cuh:647-815) + fused bias/activation.

    x [B,H,W,C], w [Co,KH,KW,Ci/groups] (depthwise: [C,KH,KW] or [C,KH,KW,1]).
    """
    if w_ohwi.dim() == 3:
        w_ohwi = w_ohwi.unsqueeze(-1)
    xn = x.permute(0, 3, 1, 2)
    wn = w_ohwi.permute(0, 3, 1, 2)
    y = F.conv2d(xn, wn, stride=tuple(stride), padding=tuple(pad), groups=groups)
    y = y.permute(0, 2, 3, 1)
    return epilogue(y, bias, None, code)


def depthwise_exact(x, w, bias, stride, pad, code):
    """Depthwise conv summed in the reference kernel's tap order (a, then b)
    with fp32 fused multiply-adds (spatial_kernels.cuh:61-90)."""
    B, H, W, C = x.shape
    KH, KW = w.shape[1], w.shape[2]
    OH = (H + 2 * pad[0] - KH) // stride[0] + 1
    OW = (W + 2 * pad[1] - KW) // stride[1] + 1
    xp = torch.zeros(B, H + 2 * pad[0], W + 2 * pad[1], C, dtype=torch.float64)
    xp[:, pad[0]:pad[0] + H, pad[1]:pad[1] + W] = x.double()
    acc = torch.zeros(B, OH, OW, C, dtype=torch.float32)
    for a in range(KH):
        for b in range(KW):
            patch = xp[:, a:a + (OH - 1) * stride[0] + 1:stride[0], b:b + (OW - 1) * stride[1] + 1:stride[1]]
            # fmaf(x, w, acc): exact product + acc, one rounding to fp32
            acc = (patch * w[:, a, b].double() + acc.double()).float()
    return epilogue(acc, bias, None, code)


def gemm(x, w, bias=None, residual=None, code=0):
    """Runtime::gemm_epilogue (runtime.cuh:514-646) / 1x1 conv: x [...,K], w [N,K]."""
    acc = x.reshape(-1, x.shape[-1]) @ w.t()
    res = residual.reshape(-1, w.shape[0]) if residual is not None else None
    return epilogue(acc, bias, res, code).reshape(*x.shape[:-1], w.shape[0])


def matmul(a, b):
    """Runtime::matmul (runtime.cuh:1013-1024): fp32 accumulate, fp16 out."""
    return rh(a @ b)


def layernorm(x, scale, bias, eps):
    """layernorm_kernel (runtime.cuh:227-261): two-pass mean/var in fp32."""
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    return rh((x - mean) * torch.rsqrt(var + eps) * scale + bias)


def softmax(x):
    """reduce_kernel softmax branch (runtime.cuh:189-225)."""
    m = x.max(-1, keepdim=True).values
    e = torch.exp(x - m)
    return rh(e / e.sum(-1, keepdim=True))


def attention(qkv, heads, dh, scale):
    """SVTR mixing attention with the unfused chain's fp16 stores:
    q' = round(q*scale); S = round(q'.k^T); P = round(softmax(S)); O = round(P.v)."""
    L, T, _ = qkv.shape
    q, k, v = qkv.reshape(L, T, 3, heads, dh).permute(2, 0, 3, 1, 4)
    q = rh(q * np.float32(scale))
    s = rh(q @ k.transpose(-1, -2))
    p = softmax(s)
    o = rh(p @ v)
    return o.permute(0, 2, 1, 3).reshape(L, T, heads * dh)


def pool_nhwc(x, k, s, pad, maximum):
    """pool_nhwc (spatial_kernels.cuh:156-193, 289-308): average excludes pad."""
    xn = x.permute(0, 3, 1, 2)
    if maximum:
        y = F.max_pool2d(xn, k, s, pad)
    else:
        y = F.avg_pool2d(xn, k, s, pad, count_include_pad=False)
    return rh(y.permute(0, 2, 3, 1))


def resize_nearest_nhwc(x, oh, ow, sh, sw, addend=None):
    """resize_nhwc_kernel (runtime.cuh:366-376): src = min(floor(dst/scale), n-1)."""
    B, H, W, C = x.shape
    rows = torch.clamp(torch.floor(torch.arange(oh, dtype=torch.float32) / np.float32(sh)).long(), max=H - 1)
    cols = torch.clamp(torch.floor(torch.arange(ow, dtype=torch.float32) / np.float32(sw)).long(), max=W - 1)
    y = x[:, rows][:, :, cols]
    if addend is not None:
        y = rh(y + addend)
    return y


def deconv_kxk(x, w, bias, code):
    """Runtime::deconv (runtime.cuh:426-453), kernel == stride, no padding.
    x [B,H,W,Ci], w [Ci,KH,KW,Co]."""
    B, H, W, Ci = x.shape
    _, KH, KW, Co = w.shape
    y = torch.einsum("bhwc,cijo->bhiwjo", x, w).reshape(B, H * KH, W * KW, Co)
    return epilogue(y, bias, None, code)


def binarize(prob: np.ndarray, thresh: float) -> np.ndarray:
    """cv::compare(pred, thresh, CMP_GT) (db_postprocess.cpp:189-190)."""
    return np.where(prob > np.float32(thresh), 255, 0).astype(np.uint8)


def argmax_prob(logits: np.ndarray):
    """Row argmax (first maximum = lowest id) and 1/sum(exp(l - max)) in float64
    (classifier.cu:456-515 semantics)."""
    l64 = logits.astype(np.float64)
    ids = l64.argmax(axis=-1).astype(np.int32)
    mx = l64.max(axis=-1)
    prob = 1.0 / np.exp(l64 - mx[..., None]).sum(axis=-1)
    return ids, prob.astype(np.float32), mx.astype(np.float32)
