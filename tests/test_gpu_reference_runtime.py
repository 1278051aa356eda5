"""Parity of the B200 layer path against the reference's OWN compiled-model
runtime, run on the same B200 (tests/ref_runtime.py: cuDNN convolutions,
cuBLAS / cuBLASLt / CUTLASS GEMMs and the reference's SIMT kernels behind
native/src/compiled/runtime.cuh, unmodified).

Each `<name>_xv` graph is written only in the exporter's vocabulary
(ppocr_b200/modelgen.py) and compiled twice from the same model.inc: against
the reference's runtime (oracle/_ref/models/<name>_xv/model.so) and against
this repository's Runtime (lib/models/<name>_xv). The fused twin
(lib/models/<name>: tcgen05 convolutions with fused epilogues, fused
attention, fused FPN steps, the depthwise + pointwise block) computes the same
function from the same seeded weights. Three comparisons per model:

  ours (exporter graph)  vs reference runtime   -- every Runtime method
  ours (fused graph)     vs reference runtime   -- the product path
  ours (fused graph)     vs ours (exporter)     -- the fusions alone

Bars: the north-star FP16 bar (max-abs 2e-2, relative L2 1e-3) everywhere.
The reference accumulates its 1x1 convolutions in FP16 (cublasGemmEx /
cuBLASLt with CUBLAS_COMPUTE_16F, or CUTLASS with a half accumulator, picked
by timing at the first enqueue: runtime.cuh:519, 654-667; cutlass_gemm.cu:
29-34) while this build accumulates in FP32, so the recognizer's K up to 2048
layers carry the reference's own rounding noise; measured on a B200: rel-L2
9.6e-4, max-abs 7.8e-3 at B=64. The FP32-oracle checks in test_gpu_models.py
and test_gpu_configs.py stay beside these.
"""

import numpy as np
import pytest
import torch

from helpers import rel_l2, rng
from ref_runtime import RefModel, ref_model_path

pytestmark = pytest.mark.gpu


def _ours(name, x_nchw, cuda, batch=None):
    from ppocr_b200 import pipeline

    m = pipeline.CompiledModel(name, cuda)
    try:
        x = torch.from_numpy(np.ascontiguousarray(x_nchw, dtype=np.float32)).to(cuda)
        out = m.output_tensor()
        stream = torch.cuda.Stream(cuda)
        m.enqueue_f32(x, out, stream)
        stream.synchronize()
        n = x.shape[0]
        return out[:n].float().cpu()
    finally:
        m.close()


def _ref(name, x_nchw, cuda):
    r = RefModel(name, cuda)
    try:
        return r.run(x_nchw)
    finally:
        r.close()


def _stats(got, want):
    d = (got.double() - want.double()).abs()
    return {"max_abs": d.max().item(), "rel_l2": rel_l2(got, want)}


def _check(report, key, got, want, max_abs, rel):
    s = _stats(got, want)
    report[key] = s
    assert torch.isfinite(got).all(), key
    assert s["max_abs"] <= max_abs and s["rel_l2"] <= rel, f"{key}: {s} (bar max_abs {max_abs}, rel_l2 {rel})"


def _need(name):
    if not ref_model_path(name).exists():
        pytest.fail(f"{ref_model_path(name)} is not built (make -C oracle ref-models)")


# Operator zoo: segments that are pure data movement, max/compare or one
# correctly rounded fp32 operation per element must be bit-identical.
_EXACT = {"pad", "pool_max", "resize", "unary0", "unary5", "binary0", "binary1", "binary2", "binary_rows",
          "transpose_0132", "slice", "nhwc", "pad_nhwc", "pool_nhwc_max", "resize_nhwc", "concat_vec8",
          "transpose_tiled", "slice3", "slice5", "concat_scalar"}


def test_operator_zoo_matches_reference(native, cuda, parity_report):
    """Every Runtime method the benchmark graphs do not use (NCHW pad / pool /
    resize / mean, the six unary modes, general-broadcast binary ops,
    transposes, slices, concats, pad_nhwc, pool_nhwc, both mean_nhwc forms,
    batched matmul) against the reference's kernels."""
    from ppocr_b200 import modelgen, models

    _need("zoo_xv")
    x = rng(70).uniform(-1, 1, modelgen.ZOO_INPUT).astype(np.float32)
    got = _ours("zoo_xv", x, cuda).reshape(-1)
    want = _ref("zoo_xv", x, cuda).reshape(-1)
    assert native.ppocr_b200_device_error() == 0
    _, _, segments = modelgen.build_zoo_xv(models.SEED)
    off = 0
    for name, shape in segments:
        n = int(np.prod(shape))
        g, w = got[off:off + n], want[off:off + n]
        off += n
        if name in _EXACT:
            assert torch.equal(g, w), f"{name}: {_stats(g, w)}"
            parity_report[f"zoo:{name}"] = {"max_abs": 0.0, "rel_l2": 0.0, "exact": True}
        else:
            _check(parity_report, f"zoo:{name}", g, w, 2e-2, 1e-3)
    assert off == got.numel()


def test_c2_block_matches_reference(native, cuda, parity_report):
    """BASELINE config 2 at full size: depthwise 5x5 (cuDNN grouped conv in
    the reference) + hardswish, pointwise 64->128 (cublasGemmEx, FP16
    accumulate over K=64) + hardswish."""
    from ppocr_b200 import workloads

    _need("block_b16_xv")
    x = workloads.c2_input(rng(71), 16).astype(np.float32).transpose(0, 3, 1, 2)
    ref = _ref("block_b16_xv", x, cuda)
    xv = _ours("block_b16_xv", x, cuda)
    fused = _ours("block_b16", x, cuda)
    assert native.ppocr_b200_device_error() == 0
    _check(parity_report, "c2:exporter_graph_vs_reference", xv, ref, 2e-2, 1e-3)
    _check(parity_report, "c2:fused_vs_reference", fused, ref, 2e-2, 1e-3)
    _check(parity_report, "c2:fused_vs_exporter_graph", fused, xv, 2e-2, 1e-3)


def test_c3_neck_matches_reference(native, cuda, parity_report):
    """BASELINE config 3 at full size: LayerNorm, linears as cuBLAS matmuls
    (FP32 compute), attention as reshape / transpose / slice / matmul /
    softmax / matmul, swish MLP, residuals."""
    from ppocr_b200 import workloads

    _need("neck_b256_xv")
    x = workloads.c3_tokens(rng(72), 256).astype(np.float32).reshape(256, 1, 40, 120)
    ref = _ref("neck_b256_xv", x, cuda)
    xv = _ours("neck_b256_xv", x, cuda)
    fused = _ours("neck_b256", x, cuda)
    assert native.ppocr_b200_device_error() == 0
    _check(parity_report, "c3:exporter_graph_vs_reference", xv, ref, 2e-2, 1e-3)
    _check(parity_report, "c3:fused_vs_reference", fused, ref, 2e-2, 1e-3)
    _check(parity_report, "c3:fused_vs_exporter_graph", fused, xv, 2e-2, 1e-3)


@pytest.mark.parametrize("name,batch", [("rec_b2", 2), ("rec_b64", 64)])
def test_recognizer_matches_reference(native, cuda, parity_report, name, batch):
    """BASELINE config 4's recognizer (backbone + neck): dense 3x3 convs in
    cuDNN, native depthwise kernels, 1x1 convs through cuBLASLt / CUTLASS
    with FP16 accumulation (K up to 2048), matmul / softmax attention."""
    _need(name + "_xv")
    x = rng(73).uniform(-1, 1, (batch, 3, 48, 320)).astype(np.float32)
    ref = _ref(name + "_xv", x, cuda)
    xv = _ours(name + "_xv", x, cuda)
    fused = _ours(name, x, cuda)
    assert native.ppocr_b200_device_error() == 0
    _check(parity_report, f"{name}:exporter_graph_vs_reference", xv, ref, 2e-2, 1e-3)
    _check(parity_report, f"{name}:fused_vs_reference", fused, ref, 2e-2, 1e-3)
    _check(parity_report, f"{name}:fused_vs_exporter_graph", fused, xv, 2e-2, 1e-3)


@pytest.mark.parametrize("name,size", [("det_b1_s128", 128), ("det_b1", 960)])
def test_detector_matches_reference(native, cuda, parity_report, name, size):
    """BASELINE config 5's DB detector on one page: cuDNN convs, FP16-
    accumulated 1x1 convs, nearest resize + add, resize + concat tail, cuDNN
    transposed convs, sigmoid, f32 output copy; binarized maps agree away
    from the threshold."""
    from oracle import layers as L

    _need(name + "_xv")
    x = rng(74).uniform(-1, 1, (1, 3, size, size)).astype(np.float32)
    ref = _ref(name + "_xv", x, cuda)
    xv = _ours(name + "_xv", x, cuda)
    fused = _ours(name if size == 128 else "det_b8", x, cuda)
    assert native.ppocr_b200_device_error() == 0
    _check(parity_report, f"{name}:exporter_graph_vs_reference", xv, ref, 2e-2, 1e-3)
    _check(parity_report, f"{name}:fused_vs_reference", fused, ref, 2e-2, 1e-3)
    _check(parity_report, f"{name}:fused_vs_exporter_graph", fused, xv, 2e-2, 1e-3)
    away = (ref - 0.3).abs() > 2e-2
    b_ref = torch.from_numpy(L.binarize(ref.numpy(), 0.3))
    b_got = torch.from_numpy(L.binarize(fused.numpy(), 0.3))
    assert torch.equal(b_got[away], b_ref[away])
    parity_report[f"{name}:binarize_agree_away_from_threshold"] = {"pixels": int(away.sum())}
