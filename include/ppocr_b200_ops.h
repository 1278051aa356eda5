// Operator-level entry points of the B200 layer path (libppocr_b200.so).
//
// Each function runs one operator of the reference's Runtime
// (native/src/compiled/runtime.cuh) on plain device pointers, with the same
// operand layouts and rounding as the Runtime method it names; the C++
// Runtime (operator API for model.inc graphs) and these functions launch the
// same kernels. Tensors are FP16 unless stated, activations NHWC, filters
// OHWI ([Co][KH][KW][Ci], the exporter's channels-last layout).
// Return 0 on success, -1 on failure (message: ppocr_b200_last_error()).
//
// Activation codes (conv, gemm, deconv): 0 bias only, 1 ReLU, 2 erf-GELU
// (runtime.cuh activation codes), and extensions 3 hardswish
// x*clamp(x/6+1/2), 4 sigmoid, 5 swish x*sigmoid(x), 6 hardsigmoid.
// Fused epilogue rounding: y = round(act(round(acc) + bias)); with a
// residual y = round(act(round(round(acc) + bias) + residual)).
#pragma once
#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Runtime::conv (runtime.cuh:647-815) for channels-last tensors: depthwise
// (groups == Ci == Co), 1x1 stride-1 GEMM, stride-1 implicit GEMM, or a
// direct convolution for small Ci (the stem). bias may be null.
int ppocr_b200_conv_nhwc(const void *x, const void *w, const void *bias,
                         void *y, int batch, int ci, int h, int w_, int co,
                         int kh, int kw, int stride_h, int stride_w, int pad_h,
                         int pad_w, int groups, int activation,
                         cudaStream_t stream);

// The stem form of Runtime::conv (runtime.cuh:766-815, cuDNN in the
// reference): 3x3 stride-2 pad-1 conv of a ci <= 4 channels-last image, run
// on the tensor cores as a 2x2 conv of the image's space-to-depth
// rearrangement. ppocr_b200_stem_s2d_pack re-lays w [co][3][3][ci] into
// wp [co][2][2][16] (co * 64 halves, 16-byte aligned) once;
// ppocr_b200_stem_conv_s2d uses caller-provided scratch of
// ppocr_b200_stem_s2d_scratch_bytes(batch, h, w) bytes (16-byte aligned).
// Output [batch][(h+1)/2][(w+1)/2][co]; bias may be null.
int ppocr_b200_stem_s2d_pack(const void *w, void *wp, int co, int ci,
                             cudaStream_t stream);
size_t ppocr_b200_stem_s2d_scratch_bytes(int batch, int h, int w_);
int ppocr_b200_stem_conv_s2d(const void *x, const void *wp, const void *bias,
                             void *y, void *scratch, int batch, int ci, int h,
                             int w_, int co, int activation,
                             cudaStream_t stream);

// Extension: the fused depthwise-separable block that Runtime builds from a
// same-size depthwise Runtime::conv (runtime.cuh:668-765) followed by the
// 1x1 Runtime::gemm_epilogue (runtime.cuh:514-646) reading its output:
// y = act_pw(x_dw . w_pw^T + b_pw), x_dw = act_dw(depthwise(x, w_dw) + b_dw)
// rounded to fp16 as the stored intermediate would be, never written to
// memory. x [batch][h][w][c], w_dw [c][k][k], w_pw [co][c],
// y [batch][h][w][co]; c == 64, k in {3, 5} (stride 1, padding k/2),
// co in {64, 128}; biases may be null (without b_dw, act_dw is not applied,
// as in the standalone depthwise form).
int ppocr_b200_dwpw_block(const void *x, const void *w_dw, const void *b_dw,
                          int act_dw, const void *w_pw, const void *b_pw,
                          int act_pw, void *y, int batch, int h, int w_,
                          int c, int k, int co, cudaStream_t stream);

// Runtime::gemm_epilogue (runtime.cuh:514-646): y[rows][co] =
// act(x[rows][ci] . w[co][ci]^T + bias) (+ residual[rows][co]).
int ppocr_b200_gemm_epilogue(const void *x, const void *w, const void *bias,
                             const void *residual, void *y, int rows, int ci,
                             int co, int activation, cudaStream_t stream);

// Runtime::matmul (runtime.cuh:1013-1024): y[b] = a[b] (m x k) . b[b] (k x n),
// contiguous batches, fp32 accumulation.
int ppocr_b200_matmul(const void *a, const void *b, void *y, int batches,
                      int m, int n, int k, cudaStream_t stream);

// Runtime::layernorm (runtime.cuh:1000-1006, kernel 227-261).
int ppocr_b200_layernorm(const void *x, const void *scale, const void *bias,
                         void *y, int rows, int cols, float epsilon,
                         cudaStream_t stream);
// Runtime::softmax (runtime.cuh:1007-1011, kernel 189-225).
int ppocr_b200_softmax(const void *x, void *y, int rows, int cols,
                       cudaStream_t stream);
// Extension: fused SVTR multi-head self-attention. qkv [lines][seq][3*H*dh]
// (q | k | v, head-major inside each), y [lines][seq][H*dh]. Matches the
// unfused matmul / scale / softmax / matmul chain of runtime.cuh:1013-1024,
// 189-225 with rounding after each step: q' = round(q*scale),
// S = round(q'.k^T), P = round(softmax(S)), O = round(P.v).
int ppocr_b200_attention(const void *qkv, void *y, int lines, int seq,
                         int heads, int head_dim, float scale,
                         cudaStream_t stream);

// Runtime::pool_nhwc (runtime.cuh:970-999): max or average (count excludes
// padding) pooling.
int ppocr_b200_pool_nhwc(const void *x, void *y, int batch, int c, int h,
                         int w, int kh, int kw, int stride_h, int stride_w,
                         int pad_h, int pad_w, int maximum,
                         cudaStream_t stream);
// Runtime::pad_nhwc (runtime.cuh:957-969): zero padding, top/left offsets.
int ppocr_b200_pad_nhwc(const void *x, void *y, int batch, int c, int h, int w,
                        int oh, int ow, int pad_h, int pad_w,
                        cudaStream_t stream);
// Runtime::resize_nearest_nhwc (runtime.cuh:461-468), asymmetric/floor;
// with a non-null addend the FPN add is fused: y = resize(x) + addend.
int ppocr_b200_resize_nearest_nhwc(const void *x, const void *addend, void *y,
                                   int batch, int c, int h, int w, int oh,
                                   int ow, float scale_h, float scale_w,
                                   cudaStream_t stream);
// Runtime::concat (runtime.cuh:901-915): y[r] = [a[r] | b[r]].
int ppocr_b200_concat(const void *a, const void *b, void *y, long long rows,
                      int na, int nb, cudaStream_t stream);
// The FPN tail of the DB detector (export.py emits it as Resize (nearest,
// runtime.cuh:461-468) per pyramid level followed by a chain of Concat ops,
// runtime.cuh:901-915) in one pass: y[n][h][w][:] = concat over k of
// srcs[k] nearest-upsampled from heights[k] x widths[k] to oh x ow (same
// asymmetric/floor mapping), channels[k] multiples of 8, 1..8 sources.
int ppocr_b200_upsample_concat_nhwc(const void *const *srcs, const int *channels,
                                    const int *heights, const int *widths, int nsrc, void *y,
                                    int batch, int oh, int ow, cudaStream_t stream);
// Runtime::transpose fast path (runtime.cuh:838-885): [batch][rows][cols] ->
// [batch][cols][rows].
int ppocr_b200_transpose(const void *x, void *y, int batch, int rows, int cols,
                         cudaStream_t stream);
// Runtime::unary (runtime.cuh:832-837): op 0 relu, 1 sigmoid, 2 hardsigmoid
// (alpha*x+beta clamped), 3 erf, 4 sqrt, 5 cast.
int ppocr_b200_unary(const void *x, void *y, long long n, int op, float alpha,
                     float beta, cudaStream_t stream);
// Runtime::binary_fast (runtime.cuh:825-831): flat broadcast indices
// (divisor, modulus) per operand; op 0 add, 1 sub, 2 mul, 3 div, 4 pow.
int ppocr_b200_binary_flat(const void *a, const void *b, void *y, long long n,
                           int a_div, int a_mod, int b_div, int b_mod, int op,
                           cudaStream_t stream);
// Runtime::mean_nhwc (runtime.cuh:937-956): global average over h*w.
int ppocr_b200_mean_nhwc(const void *x, void *y, int batch, int c, int spatial,
                         cudaStream_t stream);
// Runtime::deconv (runtime.cuh:426-453) for kernel == stride, no padding
// (the DB head's 2x2 stride-2 upsampling). w [ci][kh][kw][co]; bias may be
// null (extension: fused bias + activation).
int ppocr_b200_deconv_nhwc(const void *x, const void *w, const void *bias,
                           void *y, int batch, int h, int w_, int ci, int co,
                           int kh, int kw, int activation, cudaStream_t stream);

// The DB head's last two layers in one pass (Runtime::deconv twice,
// runtime.cuh:426-453, as export.py emits the head): y2 = act2(deconv(
// act(deconv(x, w, bias)), w2, bias2)), both 2x2 stride 2; x [batch][h][w_]
// [ci] (ci a multiple of 8), w [ci][2][2][64], bias [64] or null, w2
// [64][2][2][1], bias2 [1] or null, y2 [batch][4h][4w_][1]. Bit-identical to
// ppocr_b200_deconv_nhwc with co = 64 followed by co = 1; the 64-channel map
// is never written. Same activation codes.
int ppocr_b200_deconv_db_tail(const void *x, const void *w, const void *bias,
                              int act, const void *w2, const void *bias2,
                              int act2, void *y2, int batch, int h, int w_,
                              int ci, cudaStream_t stream);
// DB binarize (native/src/detection/db_postprocess.cpp:189-190, on device):
// map[i] = prob[i] > thresh ? 255 : 0. prob float32, map uint8.
int ppocr_b200_binarize(const float *prob, uint8_t *map, size_t n,
                        float thresh, cudaStream_t stream);
// DB post-processing front end (extension; the reference runs
// cv::findContours on the host after copying the whole FP32 map back,
// native/src/detection/db_postprocess.cpp:183-252): 8-connected components
// of `pages` binarized maps bitmap [pages][h][w] (non-zero = foreground),
// labelled 1..counts[p] per page (0 = background) into labels
// [pages][h][w] (int32) in the order OpenCV's
// connectedComponentsWithStats (connectivity 8) numbers them (each
// component's first pixel in 2x2-block raster order), with
// stats [pages][max_components][5] = (left, top, width, height, area) --
// OpenCV's layout -- and prob_sum_q32 [pages][max_components] = sum over the
// component's pixels of floor(clamp(prob, 0, 1) * 2^32) (deterministic;
// prob may be null: sums 0). Components past max_components are labelled
// and counted but get no stats (zeros). workspace: device memory of
// ppocr_b200_db_components_workspace() bytes, 256-byte aligned.
size_t ppocr_b200_db_components_workspace(int pages, int h, int w,
                                          int max_components);
int ppocr_b200_db_components(const uint8_t *bitmap, const float *prob,
                             int pages, int h, int w, int max_components,
                             int *labels, int *counts, int *stats,
                             unsigned long long *prob_sum_q32, void *workspace,
                             cudaStream_t stream);
// Frees device memory returned by ppocr_model_load_weights (cudaFree).
int ppocr_b200_device_free(void *device_pointer);
// copy_input / copy_float_output (native/src/compiled/model_library.cu:15-25).
int ppocr_b200_f32_to_f16(const float *x, void *y, size_t valid, size_t total,
                          cudaStream_t stream);
int ppocr_b200_f16_to_f32(const void *x, float *y, size_t n,
                          cudaStream_t stream);

#ifdef __cplusplus
}
#endif
