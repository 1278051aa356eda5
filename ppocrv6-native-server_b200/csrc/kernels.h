// Host-side launchers for every device kernel of the B200 layer path.
// These are the internal C++ entry points used by the Runtime (operator API),
// the model ABI shell and the extern "C" boundary in capi.cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include <string>

namespace pb2 {

// Per-device error word written by kernels whose bounded waits ran out
// (see ptx.cuh). Allocated once per device on first use; never freed.
int *device_error_word();
// Reads and clears the error word of the current device (synchronizes).
int take_device_error();
// Reads and clears the allocation-free head's timeout word (head_noalloc.cu).
int take_noalloc_error();
// Test support: writes `code` into that word (head_noalloc.cu).
cudaError_t store_noalloc_error(int code);
int sm_count();
// Sets the calling thread's message returned by ppocr_b200_last_error().
void set_last_error(const std::string &message);

// ------------------------------------------------------------ tensor cores
// Implicit-GEMM / GEMM on tcgen05. Weights are K-major: [N][taps][Ci].
// Epilogue: v = round_half(acc) + bias[n]; with a residual
// v = round_half(v) + residual[row][n]; v = act(v); y = round_half(v).
struct GemmEpilogue {
  const half *bias = nullptr;     // [N] or null
  const half *residual = nullptr; // [rows][ldr] or null
  int ldr = 0;
  half *out = nullptr; // [rows][ldo]
  int ldo = 0;
  int act = 0;
  // Nearest 2x upsampled residual (plain GEMMs): the rows are the pixels of
  // [batch][2 res_h][2 res_w] images and the residual is [batch][res_h]
  // [res_w][ldr]; output pixel (y, x) adds residual pixel (y / 2, x / 2) --
  // the FPN's resize_nearest_add_nhwc folded into the lateral 1x1 conv.
  int res_up = 0, res_h = 0, res_w = 0;
};
// Plain GEMM: out[M][N] = A[M][K] (row stride lda) x W[N][K]^T (row stride ldw).
cudaError_t tc_gemm(const half *A, int M, int K, int lda, const half *W, int N,
                    int ldw, const GemmEpilogue &epi, cudaStream_t stream);

// Stride-1 dense NHWC convolution as implicit GEMM:
// x [batch][H][W][Ci], w [Co][KH][KW][Ci], y [batch][OH][OW][Co] with
// OH = H + 2*pad_h - KH + 1, OW = W + 2*pad_w - KW + 1.
struct ConvShape {
  int batch, H, W, Ci, Co, KH, KW, pad_h, pad_w;
  // Output extent; 0 = H + 2*pad_h - KH + 1 (symmetric padding). A smaller
  // extent drops the bottom/right padding (asymmetric pad).
  int out_h = 0, out_w = 0;
};
cudaError_t tc_conv(const half *x, const half *w, const ConvShape &s,
                    const GemmEpilogue &epi, cudaStream_t stream);
// Few-channel form of tc_conv (3x3, pad 1, stride 1, Ci a multiple of 16 up
// to 64, Co a multiple of 16 up to 128, no residual): each input pixel is
// staged in shared memory once per slab of output rows and read by all nine
// taps through shifted UMMA descriptors. tc_conv routes such layers here;
// returns cudaErrorNotSupported for other shapes.
bool halo_conv_supported(const ConvShape &s, const GemmEpilogue &epi);
cudaError_t halo_conv(const half *x, const half *w, const ConvShape &s,
                      const GemmEpilogue &epi, cudaStream_t stream);
// Wide-input, narrow-output form (3x3, pad 1, stride 1, Ci a multiple of 64
// from 128 to 1024, Co a multiple of 16 up to 64, no residual): stages of R
// input rows x one 64-channel chunk, each read by the three taps of one
// filter row through shifted UMMA descriptors, with the filter streamed per
// stage. tc_conv routes such layers here.
bool halo_stream_supported(const ConvShape &s, const GemmEpilogue &epi);
cudaError_t halo_stream_conv(const half *x, const half *w, const ConvShape &s,
                             const GemmEpilogue &epi, cudaStream_t stream);

// Transposed convolution with kernel == stride (no padding) on the tensor
// cores, Co a multiple of 64: a 1x1 implicit GEMM over the input pixels with
// N = KH*KW*Co columns, each 64-column chunk (one tap's channel block) stored
// to its stride-interleaved output pixels. wpacked [KH*KW*Co][Ci] (tap-major
// rows, K-major), bias_rep [KH*KW*Co] (the bias repeated per tap) or null;
// y [batch][H*KH][W*KW][Co]. Rounding as the fused conv epilogue.
cudaError_t tc_deconv(const half *x, const half *wpacked, const half *bias_rep,
                      half *y, int batch, int H, int W, int Ci, int Co, int KH,
                      int KW, int act, cudaStream_t stream);
// The DB head's two transposed convs in one pass: tc_deconv (Ci -> 64, 2x2
// stride 2, bias_rep / act) whose fp16 outputs feed, inside the epilogue, a
// 2x2 stride-2 transposed conv 64 -> 1 (w2 fp32 [64][4] = [Ci][KH][KW],
// bias2 fp16 or null, act2) written to y2 fp16 [batch][4 H][4 W];
// bit-identical to tc_deconv followed by deconv_kxk, without the 64-channel
// map in between.
cudaError_t tc_deconv_db_tail(const half *x, const half *wpacked, const half *bias_rep, int act,
                              const float *w2, const half *bias2, int act2, half *y2, int batch,
                              int H, int W, int Ci, cudaStream_t stream);
// dst[i] = float(src[i]) (filters kept as fp32 by a fused epilogue).
cudaError_t widen_f16(const half *src, float *dst, int n, cudaStream_t stream);

// Vocabulary projection with fused row argmax / softmax-max reduction:
// logits[r][v] = hidden[r][:] . wt[v][:] + bias[v] (fp32), reduced over v to
// (max, lowest argmax, sum exp(l - max)) per vocabulary tile of 256 columns.
// Partials are laid out [tile][rows]. hidden [rows][H], wt [V][H] (K-major).
// `err_word` receives a code if a bounded wait runs out; null means the
// per-device word of device_error_word().
cudaError_t tc_vocab_partials(const half *hidden, int rows, int H,
                              const half *wt, const half *bias, int V,
                              float *part_max, int *part_id, float *part_sum,
                              int calc_prob, cudaStream_t stream,
                              int *err_word = nullptr);
int vocab_tiles(int V);
// Merges the per-tile partials into ids/prob/max_logit per row.
cudaError_t vocab_merge(const float *part_max, const int *part_id,
                        const float *part_sum, int rows, int tiles, int *ids,
                        float *prob, float *max_logit, int calc_prob,
                        cudaStream_t stream);

// Fused depthwise-separable block (C == 64, K in {3, 5}, stride 1, same
// padding; Co in {64, 128}): y = act_pw(pw(act_dw(dw(x) + bdw)) + bpw) with
// the depthwise output kept on chip. wdw [C][K][K], wpw [Co][C] (K-major),
// biases may be null (the depthwise activation then is not applied, as in
// the standalone depthwise kernels).
bool dwpw_supported(int C, int K, int Co);
cudaError_t dwpw_block(const half *x, const half *wdw, const half *bdw, int act_dw, const half *wpw,
                       const half *bpw, int act_pw, half *y, int B, int H, int W, int C, int K, int Co,
                       cudaStream_t stream);

// NHWC convolution dispatcher used by Runtime::conv and the C entry point
// (depthwise / 1x1 GEMM / implicit GEMM / direct). Weights OHWI.
cudaError_t conv_nhwc(const half *x, const half *w, const half *bias, half *y,
                      int B, int C, int H, int W, int Co, int KH, int KW,
                      int SH, int SW, int PH, int PW, int groups, int act,
                      cudaStream_t stream);

// --------------------------------------------------------------- SIMT ops
// Depthwise NHWC conv with fused bias + activation, reference rounding:
// y = round(act(round(sum) + bias)). Weights [C][KH][KW]. C % 8 == 0.
cudaError_t depthwise(const half *x, const half *w, const half *bias, half *y,
                      int batch, int C, int H, int W, int OH, int OW, int KH,
                      int KW, int SH, int SW, int PH, int PW, int act,
                      cudaStream_t stream);
// Stem 3x3 stride-2 pad-1 conv of a Ci <= 4 image on the tensor cores, as a
// 2x2 stride-1 conv of its space-to-depth rearrangement (16 channels):
// stem_s2d_pack re-lays w [Co][3][3][Ci] as wp [Co][2][2][16] (once);
// stem_conv_s2d writes the rearranged image into scratch
// (stem_s2d_scratch_bytes, 16-byte aligned) and runs the implicit GEMM.
cudaError_t stem_s2d_pack(const half *w, half *wp, int Co, int Ci,
                          cudaStream_t s);
size_t stem_s2d_scratch_bytes(int batch, int H, int W);
cudaError_t stem_conv_s2d(const half *x, const half *wp, const half *bias,
                          half *y, half *scratch, int batch, int Ci, int H,
                          int W, int Co, int act, cudaStream_t s);
// Generic NHWC direct conv for small Ci (stem): w [Co][KH][KW][Ci].
// Stem 3x3 / stride 2 / pad 1 convolution of a 3-channel NHWC image on the
// tensor cores (im2col rows built in shared memory, K = 27 -> 32).
// cudaErrorNotSupported for shapes it does not take (Co not 16/32/48/64,
// rows not a multiple of 16 bytes).
cudaError_t stem_conv_tc(const half *x, const half *w, const half *bias, half *y, int B, int H, int W, int Co,
                         int act, cudaStream_t stream);
cudaError_t direct_conv(const half *x, const half *w, const half *bias,
                        half *y, int batch, int Ci, int H, int W, int Co,
                        int OH, int OW, int KH, int KW, int SH, int SW, int PH,
                        int PW, int act, cudaStream_t stream);
cudaError_t pool_nhwc(const half *x, half *y, int batch, int C, int H, int W,
                      int OH, int OW, int KH, int KW, int SH, int SW, int PH,
                      int PW, bool maximum, cudaStream_t stream);
cudaError_t pool_nchw(const half *x, half *y, int planes, int H, int W, int OH,
                      int OW, int KH, int KW, int SH, int SW, int PH, int PW,
                      bool maximum, cudaStream_t stream);
cudaError_t pad_nhwc(const half *x, half *y, int batch, int C, int H, int W,
                     int OH, int OW, int PH, int PW, cudaStream_t stream);
cudaError_t pad_nchw(const half *x, half *y, int planes, int H, int W, int OH,
                     int OW, int PH, int PW, cudaStream_t stream);
// Nearest-neighbour resize (asymmetric coordinates, floor), optional fused add
// of `addend` (same shape as y): y = round(round(resize(x)) + addend).
// Up to kUpcatMax NHWC sources, each nearest-upsampled (resize mapping) to
// OH x OW and concatenated along channels into y (channels multiples of 8).
constexpr int kUpcatMax = 8;
struct UpcatArgs {
  const half *src[kUpcatMax];
  int C[kUpcatMax], H[kUpcatMax], W[kUpcatMax];
  float sh[kUpcatMax], sw[kUpcatMax];
  int n;
};
cudaError_t upsample_concat_nhwc(const UpcatArgs &a, half *y, int batch, int OH, int OW,
                                 cudaStream_t s);
cudaError_t resize_nearest_nhwc(const half *x, const half *addend, half *y,
                                int batch, int C, int H, int W, int OH, int OW,
                                float scale_h, float scale_w,
                                cudaStream_t stream);
cudaError_t resize_nearest_nchw(const half *x, half *y, int planes, int H,
                                int W, int OH, int OW, float scale_h,
                                float scale_w, cudaStream_t stream);
// Row-wise concat: y[r] = [a[r] (na) | b[r] (nb)].
cudaError_t concat_rows(const half *a, const half *b, half *y, long long rows,
                        int na, int nb, cudaStream_t stream);
// Batched 2D transpose: x [batch][rows][cols] -> y [batch][cols][rows].
cudaError_t transpose2d(const half *x, half *y, int batch, int rows, int cols,
                        cudaStream_t stream);
// Generic strided gather (rank <= 6): y[i] = x[offset + sum_d idx_d * stride_d].
struct Gather {
  int rank = 0;
  int shape[6] = {};
  long long stride[6] = {};
  long long offset = 0;
};
cudaError_t gather(const half *x, half *y, long long n, const Gather &g,
                   cudaStream_t stream);
// Broadcast binary: each operand indexed through its own Gather map.
cudaError_t binary(const half *a, const half *b, half *y, long long n,
                   const Gather &ga, const Gather &gb, int op,
                   cudaStream_t stream);
// Flat broadcast binary with constant divisor/modulus index maps.
cudaError_t binary_flat(const half *a, const half *b, half *y, long long n,
                        int ad, int am, int bd, int bm, int op,
                        cudaStream_t stream);
cudaError_t unary(const half *x, half *y, long long n, int op, float alpha,
                  float beta, cudaStream_t stream);
// NCHW f32 (batch rows valid, rest zero) -> NCHW fp16, the ABI input copy.
cudaError_t copy_input_f32(const float *x, half *y, size_t valid, size_t total,
                           cudaStream_t stream);
// NHWC fp16 (valid images) -> NCHW fp16 with zero tail.
cudaError_t copy_input_nhwc_f16(const half *x, half *y, int valid, int batch,
                                int C, int H, int W, cudaStream_t stream);
cudaError_t half_to_float(const half *x, float *y, size_t n,
                          cudaStream_t stream);
// ABI input staging of a layout the graph reads as is: the first `valid`
// bytes of x, zeros up to `total` bytes (16-byte vectors when aligned).
cudaError_t stage_bytes(const void *x, void *y, size_t valid, size_t total,
                        cudaStream_t stream);
// ABI output: n fp16 values copied (to_f32: widened to f32) into y, and the
// device error word `err` mirrored into host-mapped memory `err_host`
// (device pointer) by the same kernel, so that one launch replaces the output
// copy and the error-word read back.
cudaError_t output_copy(const half *x, void *y, size_t n, bool to_f32,
                        const int *err, int *err_host, cudaStream_t stream);
// NCHW f32 (valid images) -> NHWC fp16 with zero images past `valid`: the
// ABI input copy fused with the exporter's channels-last transpose.
cudaError_t nchw_f32_to_nhwc_f16(const float *x, half *y, int valid,
                                 int batch, int C, int H, int W,
                                 cudaStream_t stream);

// ------------------------------------------------------ sequence kernels
cudaError_t layernorm(const half *x, const half *scale, const half *bias,
                      half *y, int rows, int cols, float eps,
                      cudaStream_t stream);
cudaError_t softmax_rows(const half *x, half *y, int rows, int cols,
                         cudaStream_t stream);
cudaError_t mean_rows(const half *x, half *y, int rows, int cols,
                      cudaStream_t stream);
cudaError_t mean_nhwc(const half *x, half *y, int batch, int C, int spatial,
                      cudaStream_t stream);
// Batched row-major matmul y[b] = a[b] (m x k) . b[b] (k x n), fp32 accumulate.
// Batched matmul on the tensor cores with SIMT-staged operands
// (matmul_tc.cu); matmul_batched dispatches to it.
cudaError_t matmul_tc(const half *a, const half *b, half *y, int batches, int m, int n, int k, long long sa,
                      long long sb, long long sy, cudaStream_t s);
cudaError_t matmul_batched(const half *a, const half *b, half *y, int batches,
                           int m, int n, int k, long long sa, long long sb,
                           long long sy, cudaStream_t stream);
// Fused multi-head self-attention over packed qkv rows:
// qkv [lines][seq][3*heads*dh] (q | k | v), out [lines][seq][heads*dh].
// Reference rounding points: S = round(q.k^T), S = round(S*scale),
// P = round(softmax(S)), O = round(P.v).
// Tensor-core attention (attention_tc.cu) for the shapes
// attention_tc_supported() accepts; attention() dispatches to it.
bool attention_tc_supported(int seq, int dh);
cudaError_t attention_tc(const half *qkv, half *out, int lines, int seq, int heads, int dh, float scale,
                         cudaStream_t s);
// SIMT attention kernels (seq.cu), used for every other shape.
cudaError_t attention_simt(const half *qkv, half *out, int lines, int seq, int heads, int dh, float scale,
                           cudaStream_t s);
cudaError_t attention(const half *qkv, half *out, int lines, int seq, int heads,
                      int dh, float scale, cudaStream_t stream);

// ----------------------------------------------------------- head kernels
// Row argmax / softmax-max over fp16 logits [rows][V].
cudaError_t logits_argmax_prob(const half *logits, int rows, int V, int *ids,
                               float *prob, float *max_logit, int calc_prob,
                               cudaStream_t stream);
// CTC greedy collapse per line: drop repeats, then blanks; mean kept prob.
// out_ids [lines][T] (compacted, -1 padded), out_len [lines], out_score.
cudaError_t ctc_collapse(const int *ids, const float *probs, int lines, int T,
                         int blank, int *out_ids, int *out_len,
                         float *out_score, cudaStream_t stream);
// Transpose W [H][V] -> wt [V][H] (K-major) for the vocabulary projection.
cudaError_t pack_vocab_weight(const half *w, half *wt, int H, int V,
                              cudaStream_t stream);
// p(class)/(p(class)+p(max)) for one selected class.
cudaError_t selected_class_vs_max(const half *hidden, const half *w,
                                  const half *bias, const float *max_logits,
                                  float *out, int rows, int H, int V,
                                  int class_id, cudaStream_t stream);

// ------------------------------------------------------- detector kernels
// DB post-processing front end: 8-connected component labelling of
// binarized maps with (left, top, width, height, area) and fixed-point
// probability sums per component (see ppocr_b200_db_components).
size_t db_components_workspace(int pages, int H, int W, int max_comp);
cudaError_t db_components(const uint8_t *bitmap, const float *prob, int pages, int H, int W, int max_comp,
                          int *labels, int *counts, int *stats, unsigned long long *probq, void *workspace,
                          cudaStream_t stream);
// DB binarize: map[i] = prob[i] > thresh ? 255 : 0.
cudaError_t binarize(const float *prob, uint8_t *map, size_t n, float thresh,
                     cudaStream_t stream);
// Transposed conv, kernel == stride, no padding (DB head 2x2 s2):
// x [batch][H][W][Ci], w [Ci][KH][KW][Co], y [batch][H*KH][W*KW][Co].
// Packs a [Ci][KH][KW][Co] transposed-conv filter for tc_deconv
// ([KH*KW*Co][Ci]) and repeats the bias per tap (bias may be null).
cudaError_t deconv_pack(const half *w, const half *bias, half *wpacked,
                        half *bias_rep, int Ci, int Co, int KH, int KW,
                        cudaStream_t s);
cudaError_t deconv_kxk(const half *x, const half *w, const half *bias, half *y,
                       int batch, int H, int W, int Ci, int Co, int KH, int KW,
                       int act, cudaStream_t stream);

// -------------------------------------------------- page / line preprocess
// One decoded RGB line image of a line-tensor batch (host-computed layout).
struct LineGeo {
  long long offset;   // byte offset of the image in the pixel buffer
  int width, height;  // source size
  int stride;         // bytes per source row
  int resized_width;  // ceil(48 * width / height) <= bucket
  float scale_x, scale_y;
  int copy;           // 48-high line of exactly resized_width: no resampling
};
constexpr int kMaxLineBatch = 512; // lines per launch (kernel parameter space)
struct LineBatch {
  LineGeo line[kMaxLineBatch];
};
// Line tensors [lines][48][bucket][3] fp16 (PREP_F16_NHWC) or
// [lines][3][48][bucket] f32 (PREP_F32_NCHW) from the images of `lb`.
cudaError_t line_tensors(const uint8_t *pixels, const LineBatch &lb, int lines, void *out, int bucket, int fmt,
                         cudaStream_t stream);
// Output formats of the preprocessing kernels.
enum PrepFormat { PREP_F32_NCHW = 0, PREP_F16_NHWC = 1 };
// Detector resize + normalize of `images` u8 HWC (3-channel) pages, each
// src_h x src_w with row pitch src_step bytes, image i at
// src + i * src_image_bytes, into [images][3][dst_h][dst_w] f32 or
// [images][dst_h][dst_w][3] fp16; content_h x content_w is the resized
// page's rectangle, the rest of the canvas is white.
cudaError_t detector_preprocess(const uint8_t *src, int src_h, int src_w,
                                long long src_step, long long src_image_bytes,
                                int images, void *dst, int dst_h, int dst_w,
                                int content_h, int content_w, int source_is_bgr,
                                int fmt, cudaStream_t stream);
// Batched perspective ROI warp of one u8 HWC page: crop b samples the page
// at m_invs[9b..9b+8] (inverse homography, row-major 3x3) for x <
// crop_widths[b]; [batch][3][dst_h][dst_w] f32 or [batch][dst_h][dst_w][3]
// fp16, values v/127.5 - 1.
cudaError_t roi_warp(const uint8_t *src, int src_h, int src_w, long long src_step,
                     const float *m_invs, const int *crop_widths, void *dst,
                     int batch, int dst_h, int dst_w, int out_bgr, int fmt,
                     cudaStream_t stream);

} // namespace pb2
