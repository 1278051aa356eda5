// extern "C" boundary of libppocr_b200.so: the head API
// (include/ppocr_b200_head.h) and the operator-level entry points
// (include/ppocr_b200_ops.h). Thin argument checks + kernels.h launchers.
#include "../../include/ppocr_b200_head.h"
#include "../../include/ppocr_b200_ops.h"
#include "../../include/ppocr_b200_preprocess.h"
#include "kernels.h"
#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <utility>

using namespace pb2;

namespace {
thread_local std::string g_error;

int fail(const std::string &msg) {
  g_error = msg;
  return -1;
}
int status(cudaError_t e, const char *what) {
  if (e == cudaSuccess)
    return 0;
  return fail(std::string(what) + ": " + cudaGetErrorString(e));
}
const half *H(const void *p) { return static_cast<const half *>(p); }
half *Hm(void *p) { return static_cast<half *>(p); }

// Workspace of the reference-signature head, one per (device, stream): the
// per-call transposed weight and, when the caller's partial buffers are sized
// for the reference's vocabulary tiles (fewer than the 256-column tiles this
// kernel reduces), the partials. Work on one stream is ordered, so a stream's
// buffer is reused without synchronisation; growing it frees the old buffer
// in stream order (cudaFreeAsync), after the work already queued on that
// stream. Callers on different streams never share a buffer, and nothing
// persists between calls but the allocation: each call repacks the weight
// it is given, so results depend only on that call's arguments.
struct StreamWorkspace {
  void *ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_ws_mutex;
std::map<std::pair<int, cudaStream_t>, StreamWorkspace> g_ws;

void *stream_workspace(size_t bytes, cudaStream_t stream) {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess)
    return nullptr;
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  StreamWorkspace &w = g_ws[{d, stream}];
  if (w.bytes < bytes) {
    if (w.ptr)
      cudaFreeAsync(w.ptr, stream);
    w.ptr = nullptr;
    w.bytes = 0;
    if (cudaMallocAsync(&w.ptr, bytes, stream) != cudaSuccess)
      return nullptr;
    w.bytes = bytes;
  }
  return w.ptr;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
} // namespace

void pb2::set_last_error(const std::string &message) { g_error = message; }

extern "C" {

const char *ppocr_b200_last_error(void) { return g_error.c_str(); }

int ppocr_b200_device_error(void) {
  cudaDeviceSynchronize();
  // Both words are read (and so cleared); the library-wide one is reported
  // first when both hold a code.
  const int shared = take_device_error();
  const int noalloc = take_noalloc_error();
  return shared ? shared : noalloc;
}

int ppocr_b200_test_store_error_code(int which, int code) {
  g_error.clear();
  if (which == 0) {
    int *word = device_error_word();
    if (!word)
      return fail("cannot allocate the device error word");
    return status(cudaMemcpy(word, &code, sizeof(int), cudaMemcpyHostToDevice),
                  "store error code");
  }
  if (which == 1)
    return status(store_noalloc_error(code), "store allocation-free error code");
  return fail("which must be 0 (library word) or 1 (allocation-free head word)");
}

int ppocr_b200_classifier_workspace(int rows, int vocab, int row_block,
                                    int vocab_tile, int *num_row_blocks,
                                    int *num_vocab_blocks,
                                    size_t *partial_count) {
  g_error.clear();
  if (!num_row_blocks || !num_vocab_blocks || !partial_count)
    return fail("null output pointer");
  if (rows <= 0 || vocab <= 0) {
    *num_row_blocks = *num_vocab_blocks = 0;
    *partial_count = 0;
    return 0;
  }
  if (row_block <= 0 || row_block > 16 || vocab_tile <= 0)
    return fail("invalid tiled classifier workspace shape");
  // The reference's shape, unchanged (classifier.cu:520-536), so buffers
  // sized by either library fit ppocr_b200_linear_argmax_prob.
  *num_row_blocks = (rows + row_block - 1) / row_block;
  *num_vocab_blocks = (vocab + vocab_tile - 1) / vocab_tile;
  *partial_count = static_cast<size_t>(*num_row_blocks) *
                   static_cast<size_t>(*num_vocab_blocks) *
                   static_cast<size_t>(row_block);
  return 0;
}

int ppocr_b200_classifier_pack(const void *weight, void *packed, int hidden,
                               int vocab, cudaStream_t stream) {
  g_error.clear();
  if (!weight || !packed || hidden <= 0 || vocab <= 0)
    return fail("invalid classifier pack arguments");
  return status(pack_vocab_weight(H(weight), Hm(packed), hidden, vocab, stream),
                "classifier pack");
}

int ppocr_b200_classifier_run_packed(
    const void *hidden, const void *packed, const void *bias, int *ids,
    float *prob, float *max_logits, int rows, int hidden_size, int vocab,
    int *part_id, float *part_max, float *part_sum, int calc_prob,
    cudaStream_t stream) {
  g_error.clear();
  if (rows <= 0)
    return 0;
  if (!hidden || !packed || !bias || !ids || !prob || !max_logits ||
      !part_id || !part_max || !part_sum || hidden_size <= 0 ||
      hidden_size % 8 || vocab <= 0)
    return fail("invalid classifier launch arguments");
  cudaError_t e = tc_vocab_partials(H(hidden), rows, hidden_size, H(packed),
                                    H(bias), vocab, part_max, part_id, part_sum,
                                    calc_prob, stream);
  if (e != cudaSuccess)
    return status(e, "vocab projection");
  return status(vocab_merge(part_max, part_id, part_sum, rows,
                            vocab_tiles(vocab), ids, prob, max_logits,
                            calc_prob, stream),
                "vocab merge");
}

int ppocr_b200_linear_argmax_prob(
    const void *hidden, const void *weight, const void *bias, int *ids,
    float *prob, float *max_logits, int rows, int hidden_size, int vocab,
    int vocab_tile, int *part_id, float *part_max, float *part_sum,
    int calc_prob, cudaStream_t stream) {
  g_error.clear();
  if (rows <= 0)
    return 0;
  // Same rejections as classifier.cu:619-623 (H % 16, tile % 16, buffers).
  if (hidden_size <= 0 || vocab <= 0 || hidden_size % 16 != 0 ||
      vocab_tile <= 0 || vocab_tile % 16 != 0 || !part_id || !part_max ||
      !part_sum || !hidden || !weight || !bias)
    return fail("invalid WMMA classifier launch arguments");
  // The caller sized the partials for the reference's WMMA path: 16-row
  // blocks x ceil(vocab / vocab_tile) tiles (classifier.cu:624-625). This
  // kernel needs rows x ceil(vocab / 256); when that does not fit, the
  // partials go to the stream's workspace instead.
  const size_t need = static_cast<size_t>(rows) * vocab_tiles(vocab);
  const size_t have = round_up(static_cast<size_t>(rows), 16) *
                      ((static_cast<size_t>(vocab) + vocab_tile - 1) / vocab_tile);
  const size_t pack_bytes = round_up(static_cast<size_t>(hidden_size) * vocab * 2, 256);
  const size_t part_bytes = have >= need ? 0 : round_up(need * 4, 256);
  auto *ws = static_cast<unsigned char *>(stream_workspace(pack_bytes + 3 * part_bytes, stream));
  if (!ws)
    return fail("cannot allocate the classifier workspace");
  half *packed = reinterpret_cast<half *>(ws);
  if (part_bytes) {
    part_max = reinterpret_cast<float *>(ws + pack_bytes);
    part_id = reinterpret_cast<int *>(ws + pack_bytes + part_bytes);
    part_sum = reinterpret_cast<float *>(ws + pack_bytes + 2 * part_bytes);
  }
  cudaError_t e = pack_vocab_weight(H(weight), packed, hidden_size, vocab, stream);
  if (e != cudaSuccess)
    return status(e, "classifier pack");
  return ppocr_b200_classifier_run_packed(hidden, packed, bias, ids, prob,
                                          max_logits, rows, hidden_size, vocab,
                                          part_id, part_max, part_sum,
                                          calc_prob, stream);
}

int ppocr_b200_selected_class_vs_max_probability(
    const void *hidden, const void *weight, const void *bias,
    const float *max_logits, float *out, int rows, int hidden_size, int vocab,
    int class_id, cudaStream_t stream) {
  g_error.clear();
  if (rows <= 0)
    return 0;
  if (!hidden || !weight || !bias || !max_logits || !out || hidden_size <= 0 ||
      vocab <= 0 || class_id < 0 || class_id >= vocab)
    return fail("invalid selected-class classifier launch arguments");
  return status(selected_class_vs_max(H(hidden), H(weight), H(bias), max_logits,
                                      out, rows, hidden_size, vocab, class_id,
                                      stream),
                "selected class");
}

int ppocr_b200_logits_argmax_prob(const void *logits, int rows, int vocab,
                                  int *ids, float *prob, float *max_logits,
                                  int calc_prob, cudaStream_t stream) {
  g_error.clear();
  if (rows <= 0)
    return 0;
  if (!logits || !ids || !prob || !max_logits || vocab <= 0)
    return fail("invalid logits argmax arguments");
  return status(logits_argmax_prob(H(logits), rows, vocab, ids, prob,
                                   max_logits, calc_prob, stream),
                "logits argmax");
}

int ppocr_b200_ctc_collapse(const int *ids, const float *probs, int lines,
                            int T, int blank, int *out_ids, int *out_len,
                            float *out_score, cudaStream_t stream) {
  g_error.clear();
  if (lines < 0 || T < 0)
    return fail("batch_size and seq_len must be non-negative");
  if (lines == 0 || T == 0) {
    if (lines > 0 && out_len && out_score) {
      cudaMemsetAsync(out_len, 0, sizeof(int) * lines, stream);
      cudaMemsetAsync(out_score, 0, sizeof(float) * lines, stream);
    }
    return 0;
  }
  if (!ids || !out_ids || !out_len || !out_score)
    return fail("null collapse buffer");
  return status(ctc_collapse(ids, probs, lines, T, blank, out_ids, out_len,
                             out_score, stream),
                "ctc collapse");
}

// ------------------------------------------------------------- operators
int ppocr_b200_conv_nhwc(const void *x, const void *w, const void *bias,
                         void *y, int batch, int ci, int h, int w_, int co,
                         int kh, int kw, int sh, int sw, int ph, int pw,
                         int groups, int act, cudaStream_t stream) {
  g_error.clear();
  if (!x || !w || !y || batch <= 0 || ci <= 0 || co <= 0 || kh <= 0 ||
      kw <= 0 || sh <= 0 || sw <= 0 || ph < 0 || pw < 0 || groups <= 0)
    return fail("invalid conv arguments");
  const int oh = (h + 2 * ph - kh) / sh + 1, ow = (w_ + 2 * pw - kw) / sw + 1;
  if (oh <= 0 || ow <= 0)
    return fail("conv output is empty");
  cudaError_t e = conv_nhwc(H(x), H(w), H(bias), Hm(y), batch, ci, h, w_, co,
                            kh, kw, sh, sw, ph, pw, groups, act, stream);
  if (e == cudaErrorNotSupported)
    return fail("unsupported conv form");
  return status(e, "conv");
}

int ppocr_b200_stem_s2d_pack(const void *w, void *wp, int co, int ci,
                             cudaStream_t stream) {
  g_error.clear();
  if (!w || !wp || co <= 0 || co % 8 || ci <= 0 || ci > 4)
    return fail("invalid stem pack arguments");
  return status(stem_s2d_pack(H(w), Hm(wp), co, ci, stream), "stem pack");
}

size_t ppocr_b200_stem_s2d_scratch_bytes(int batch, int h, int w_) {
  if (batch <= 0 || h <= 0 || w_ <= 0)
    return 0;
  return stem_s2d_scratch_bytes(batch, h, w_);
}

int ppocr_b200_stem_conv_s2d(const void *x, const void *wp, const void *bias,
                             void *y, void *scratch, int batch, int ci, int h,
                             int w_, int co, int act, cudaStream_t stream) {
  g_error.clear();
  if (!x || !wp || !y || !scratch || batch <= 0 || h <= 0 || w_ <= 0 ||
      ci <= 0 || ci > 4 || co <= 0 || co % 8)
    return fail("invalid stem conv arguments");
  if ((reinterpret_cast<uintptr_t>(scratch) | reinterpret_cast<uintptr_t>(wp) |
       reinterpret_cast<uintptr_t>(y)) & 15)
    return fail("stem conv buffers must be 16-byte aligned");
  return status(stem_conv_s2d(H(x), H(wp), H(bias), Hm(y), Hm(scratch), batch, ci, h, w_,
                              co, act, stream),
                "stem conv");
}

int ppocr_b200_gemm_epilogue(const void *x, const void *w, const void *bias,
                             const void *residual, void *y, int rows, int ci,
                             int co, int act, cudaStream_t stream) {
  g_error.clear();
  if (!x || !w || !y || rows < 0 || ci <= 0 || co <= 0 || ci % 8 || co % 8)
    return fail("invalid gemm_epilogue arguments");
  GemmEpilogue e;
  e.bias = H(bias);
  e.residual = H(residual);
  e.ldr = co;
  e.out = Hm(y);
  e.ldo = co;
  e.act = act;
  return status(tc_gemm(H(x), rows, ci, ci, H(w), co, ci, e, stream), "gemm");
}

int ppocr_b200_matmul(const void *a, const void *b, void *y, int batches,
                      int m, int n, int k, cudaStream_t stream) {
  g_error.clear();
  // Empty operands (k = 0) may be null: the product is zeros.
  if ((k > 0 && (!a || !b)) || !y || batches < 0 || m < 0 || n < 0 || k < 0)
    return fail("invalid matmul arguments");
  return status(matmul_batched(H(a), H(b), Hm(y), batches, m, n, k,
                               static_cast<long long>(m) * k,
                               static_cast<long long>(k) * n,
                               static_cast<long long>(m) * n, stream),
                "matmul");
}

int ppocr_b200_layernorm(const void *x, const void *scale, const void *bias,
                         void *y, int rows, int cols, float eps,
                         cudaStream_t stream) {
  g_error.clear();
  if (!x || !scale || !bias || !y || rows < 0 || cols <= 0)
    return fail("invalid layernorm arguments");
  return status(layernorm(H(x), H(scale), H(bias), Hm(y), rows, cols, eps,
                          stream),
                "layernorm");
}

int ppocr_b200_softmax(const void *x, void *y, int rows, int cols,
                       cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || rows < 0 || cols <= 0)
    return fail("invalid softmax arguments");
  return status(softmax_rows(H(x), Hm(y), rows, cols, stream), "softmax");
}

int ppocr_b200_attention(const void *qkv, void *y, int lines, int seq,
                         int heads, int dh, float scale, cudaStream_t stream) {
  g_error.clear();
  if (!qkv || !y || lines < 0 || seq <= 0 || heads <= 0 || dh <= 0)
    return fail("invalid attention arguments");
  cudaError_t e = attention(H(qkv), Hm(y), lines, seq, heads, dh, scale, stream);
  if (e == cudaErrorInvalidValue)
    return fail("attention line does not fit in shared memory");
  return status(e, "attention");
}

int ppocr_b200_pool_nhwc(const void *x, void *y, int batch, int c, int h,
                         int w, int kh, int kw, int sh, int sw, int ph, int pw,
                         int maximum, cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || batch <= 0 || c <= 0 || kh <= 0 || kw <= 0 || sh <= 0 ||
      sw <= 0)
    return fail("invalid pool arguments");
  const int oh = (h + 2 * ph - kh) / sh + 1, ow = (w + 2 * pw - kw) / sw + 1;
  return status(pool_nhwc(H(x), Hm(y), batch, c, h, w, oh, ow, kh, kw, sh, sw,
                          ph, pw, maximum != 0, stream),
                "pool");
}

int ppocr_b200_pad_nhwc(const void *x, void *y, int batch, int c, int h, int w,
                        int oh, int ow, int ph, int pw, cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || batch <= 0 || c <= 0)
    return fail("invalid pad arguments");
  return status(pad_nhwc(H(x), Hm(y), batch, c, h, w, oh, ow, ph, pw, stream),
                "pad");
}

int ppocr_b200_resize_nearest_nhwc(const void *x, const void *addend, void *y,
                                   int batch, int c, int h, int w, int oh,
                                   int ow, float sh, float sw,
                                   cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || batch <= 0 || c <= 0 || sh <= 0 || sw <= 0)
    return fail("invalid resize arguments");
  return status(resize_nearest_nhwc(H(x), H(addend), Hm(y), batch, c, h, w, oh,
                                    ow, sh, sw, stream),
                "resize");
}

int ppocr_b200_concat(const void *a, const void *b, void *y, long long rows,
                      int na, int nb, cudaStream_t stream) {
  g_error.clear();
  if (!a || !b || !y || rows < 0 || na < 0 || nb < 0)
    return fail("invalid concat arguments");
  return status(concat_rows(H(a), H(b), Hm(y), rows, na, nb, stream), "concat");
}

int ppocr_b200_upsample_concat_nhwc(const void *const *srcs, const int *channels,
                                    const int *heights, const int *widths, int nsrc, void *y,
                                    int batch, int oh, int ow, cudaStream_t stream) {
  g_error.clear();
  if (!srcs || !channels || !heights || !widths || !y || nsrc < 1 || nsrc > kUpcatMax ||
      batch < 0 || oh <= 0 || ow <= 0)
    return fail("invalid upsample_concat arguments");
  UpcatArgs a{};
  a.n = nsrc;
  for (int k = 0; k < nsrc; ++k) {
    if (heights[k] <= 0 || widths[k] <= 0)
      return fail("invalid upsample_concat source size");
    a.src[k] = H(srcs[k]);
    a.C[k] = channels[k];
    a.H[k] = heights[k];
    a.W[k] = widths[k];
    a.sh[k] = static_cast<float>(oh) / heights[k];
    a.sw[k] = static_cast<float>(ow) / widths[k];
  }
  return status(upsample_concat_nhwc(a, Hm(y), batch, oh, ow, stream), "upsample_concat");
}

int ppocr_b200_transpose(const void *x, void *y, int batch, int rows, int cols,
                         cudaStream_t stream) {
  g_error.clear();
  if (!x || !y)
    return fail("invalid transpose arguments");
  return status(transpose2d(H(x), Hm(y), batch, rows, cols, stream),
                "transpose");
}

int ppocr_b200_unary(const void *x, void *y, long long n, int op, float alpha,
                     float beta, cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || n < 0 || op < 0 || op > 5)
    return fail("invalid unary arguments");
  return status(unary(H(x), Hm(y), n, op, alpha, beta, stream), "unary");
}

int ppocr_b200_binary_flat(const void *a, const void *b, void *y, long long n,
                           int ad, int am, int bd, int bm, int op,
                           cudaStream_t stream) {
  g_error.clear();
  if (!a || !b || !y || n < 0 || op < 0 || op > 4 || ad <= 0 || bd <= 0)
    return fail("invalid binary arguments");
  return status(binary_flat(H(a), H(b), Hm(y), n, ad, am, bd, bm, op, stream),
                "binary");
}

int ppocr_b200_mean_nhwc(const void *x, void *y, int batch, int c, int spatial,
                         cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || batch < 0 || c <= 0 || spatial <= 0)
    return fail("invalid mean arguments");
  return status(mean_nhwc(H(x), Hm(y), batch, c, spatial, stream), "mean");
}

int ppocr_b200_deconv_nhwc(const void *x, const void *w, const void *bias,
                           void *y, int batch, int h, int w_, int ci, int co,
                           int kh, int kw, int act, cudaStream_t stream) {
  g_error.clear();
  if (!x || !w || !y || batch < 0 || ci <= 0 || co <= 0 || kh <= 0 || kw <= 0)
    return fail("invalid deconv arguments");
  if (co % 64 == 0 && ci % 8 == 0) {
    // Tensor-core path: pack the filter (and repeat the bias) into
    // stream-ordered temporaries, released on the same stream.
    const size_t wn = static_cast<size_t>(ci) * kh * kw * co;
    void *wp = nullptr, *bp = nullptr;
    cudaError_t e = cudaMallocAsync(&wp, wn * 2, stream);
    if (e == cudaSuccess && bias)
      e = cudaMallocAsync(&bp, static_cast<size_t>(kh) * kw * co * 2, stream);
    if (e == cudaSuccess)
      e = deconv_pack(H(w), H(bias), static_cast<half *>(wp), static_cast<half *>(bp), ci, co,
                      kh, kw, stream);
    if (e == cudaSuccess)
      e = tc_deconv(H(x), static_cast<half *>(wp), static_cast<half *>(bp), Hm(y), batch, h,
                    w_, ci, co, kh, kw, act, stream);
    if (wp)
      cudaFreeAsync(wp, stream);
    if (bp)
      cudaFreeAsync(bp, stream);
    return status(e, "deconv");
  }
  return status(deconv_kxk(H(x), H(w), H(bias), Hm(y), batch, h, w_, ci, co,
                           kh, kw, act, stream),
                "deconv");
}

int ppocr_b200_deconv_db_tail(const void *x, const void *w, const void *bias,
                              int act, const void *w2, const void *bias2,
                              int act2, void *y2, int batch, int h, int w_,
                              int ci, cudaStream_t stream) {
  g_error.clear();
  if (!x || !w || !w2 || !y2 || batch < 0 || h <= 0 || w_ <= 0 || ci <= 0 || ci % 8)
    return fail("invalid deconv_db_tail arguments");
  // Packed first filter, repeated bias and the fp32 second filter in
  // stream-ordered temporaries, released on the same stream.
  const size_t wn = static_cast<size_t>(ci) * 4 * 64;
  void *wp = nullptr, *bp = nullptr, *w2f = nullptr;
  cudaError_t e = cudaMallocAsync(&wp, wn * 2, stream);
  if (e == cudaSuccess && bias)
    e = cudaMallocAsync(&bp, 4 * 64 * 2, stream);
  if (e == cudaSuccess)
    e = cudaMallocAsync(&w2f, 256 * sizeof(float), stream);
  if (e == cudaSuccess)
    e = deconv_pack(H(w), H(bias), static_cast<half *>(wp), static_cast<half *>(bp), ci, 64, 2, 2, stream);
  if (e == cudaSuccess)
    e = widen_f16(H(w2), static_cast<float *>(w2f), 256, stream);
  if (e == cudaSuccess)
    e = tc_deconv_db_tail(H(x), static_cast<half *>(wp), static_cast<half *>(bp), act,
                          static_cast<float *>(w2f), H(bias2), act2, Hm(y2), batch, h, w_, ci, stream);
  for (void *p : {wp, bp, w2f})
    if (p)
      cudaFreeAsync(p, stream);
  return status(e, "deconv_db_tail");
}

int ppocr_b200_dwpw_block(const void *x, const void *w_dw, const void *b_dw,
                          int act_dw, const void *w_pw, const void *b_pw,
                          int act_pw, void *y, int batch, int h, int w_,
                          int c, int k, int co, cudaStream_t stream) {
  g_error.clear();
  if (!x || !w_dw || !w_pw || !y || batch < 0 || h < 0 || w_ < 0)
    return fail("invalid dwpw block arguments");
  if (!dwpw_supported(c, k, co))
    return fail("dwpw block supports c == 64, k in {3, 5}, co in {64, 128}");
  return status(dwpw_block(H(x), H(w_dw), H(b_dw), act_dw, H(w_pw), H(b_pw),
                           act_pw, Hm(y), batch, h, w_, c, k, co, stream),
                "dwpw block");
}

int ppocr_b200_binarize(const float *prob, uint8_t *map, size_t n, float thresh,
                        cudaStream_t stream) {
  g_error.clear();
  if (!prob || !map)
    return fail("invalid binarize arguments");
  return status(binarize(prob, map, n, thresh, stream), "binarize");
}

int ppocr_b200_detector_preprocess(const void *src, size_t src_step,
                                   int src_rows, int src_cols,
                                   size_t src_image_bytes, int images,
                                   void *dst, int dst_h, int dst_w,
                                   int content_h, int content_w,
                                   int source_is_bgr, int format,
                                   cudaStream_t stream) {
  g_error.clear();
  if (content_h <= 0 || content_w <= 0 || content_h > dst_h ||
      content_w > dst_w || src == nullptr || src_rows <= 0 || src_cols <= 0 ||
      src_step < static_cast<size_t>(src_cols) * 3 || dst == nullptr ||
      dst_h <= 0 || dst_w <= 0 || images < 0 ||
      (images > 1 && src_image_bytes < src_step * src_rows) ||
      (format != PPOCR_B200_PREP_F32_NCHW && format != PPOCR_B200_PREP_F16_NHWC))
    return fail("invalid detector preprocess arguments");
  return status(detector_preprocess(static_cast<const uint8_t *>(src), src_rows,
                                    src_cols, static_cast<long long>(src_step),
                                    static_cast<long long>(src_image_bytes),
                                    images, dst, dst_h, dst_w, content_h,
                                    content_w, source_is_bgr ? 1 : 0, format,
                                    stream),
                "detector preprocess");
}

int ppocr_b200_resize_normalize_detector_padded(
    const void *src, size_t src_step, int src_rows, int src_cols,
    float *dst_nchw, int dst_h, int dst_w, int content_h, int content_w,
    int source_is_bgr, cudaStream_t stream) {
  return ppocr_b200_detector_preprocess(src, src_step, src_rows, src_cols, 0, 1,
                                        dst_nchw, dst_h, dst_w, content_h,
                                        content_w, source_is_bgr,
                                        PPOCR_B200_PREP_F32_NCHW, stream);
}

int ppocr_b200_resize_normalize_detector(const void *src, size_t src_step,
                                         int src_rows, int src_cols,
                                         float *dst_nchw, int dst_h, int dst_w,
                                         int source_is_bgr,
                                         cudaStream_t stream) {
  return ppocr_b200_resize_normalize_detector_padded(
      src, src_step, src_rows, src_cols, dst_nchw, dst_h, dst_w, dst_h, dst_w,
      source_is_bgr, stream);
}

int ppocr_b200_roi_warp(const void *src, size_t src_step, int src_rows,
                        int src_cols, const float *d_m_invs,
                        const int *d_crop_widths, void *dst, int batch,
                        int dst_h, int dst_w, int output_bgr, int format,
                        cudaStream_t stream) {
  g_error.clear();
  if (batch <= 0)
    return 0;
  if (src == nullptr || src_rows <= 0 || src_cols <= 0 ||
      src_step < static_cast<size_t>(src_cols) * 3 || !d_m_invs ||
      !d_crop_widths || !dst || dst_h < 0 || dst_w < 0 ||
      (format != PPOCR_B200_PREP_F32_NCHW && format != PPOCR_B200_PREP_F16_NHWC))
    return fail("invalid roi warp arguments");
  return status(roi_warp(static_cast<const uint8_t *>(src), src_rows, src_cols,
                         static_cast<long long>(src_step), d_m_invs,
                         d_crop_widths, dst, batch, dst_h, dst_w,
                         output_bgr ? 1 : 0, format, stream),
                "roi warp");
}

int ppocr_b200_line_tensors(const void *pixels, const long long *offsets,
                            const int *widths, const int *heights,
                            const int *strides, int lines, int bucket,
                            void *out, int format, cudaStream_t stream) {
  g_error.clear();
  if (lines < 0 || bucket <= 0 || (lines > 0 && (!pixels || !offsets || !widths || !heights || !strides || !out)) ||
      (format != PPOCR_B200_PREP_F32_NCHW && format != PPOCR_B200_PREP_F16_NHWC))
    return fail("invalid line tensor arguments");
  const size_t elem = format == PPOCR_B200_PREP_F16_NHWC ? 2 : 4;
  for (int c0 = 0; c0 < lines; c0 += kMaxLineBatch) {
    const int n = std::min(kMaxLineBatch, lines - c0);
    static thread_local LineBatch lb;
    for (int k = 0; k < n; ++k) {
      const int i = c0 + k;
      const int w = widths[i], h = heights[i];
      if (w <= 0 || h <= 0)
        return fail("line dimensions must be positive");
      if (strides[i] < 3 * w || offsets[i] < 0)
        return fail("invalid line tensor arguments");
      const long long natural = (static_cast<long long>(w) * 48 + h - 1) / h;
      if (natural > bucket)
        return fail("line normalized width " + std::to_string(natural) + " exceeds maximum " +
                    std::to_string(bucket) + "; split the line crop");
      LineGeo &g = lb.line[k];
      g.offset = offsets[i];
      g.width = w;
      g.height = h;
      g.stride = strides[i];
      g.resized_width = static_cast<int>(natural);
      g.scale_x = static_cast<float>(w) / static_cast<float>(natural);
      g.scale_y = static_cast<float>(h) / 48.0f;
      g.copy = (w == natural && h == 48) ? 1 : 0;
    }
    void *dst = static_cast<char *>(out) + static_cast<size_t>(c0) * 3 * 48 * bucket * elem;
    const int st = status(line_tensors(static_cast<const uint8_t *>(pixels), lb, n, dst, bucket, format, stream),
                          "line tensors");
    if (st)
      return st;
  }
  return 0;
}

int ppocr_b200_batch_roi_warp(const void *src, size_t src_step, int src_rows,
                              int src_cols, const float *d_m_invs,
                              const int *d_crop_widths, float *d_dst_batch,
                              int batch, int dst_h, int dst_w, int output_bgr,
                              cudaStream_t stream) {
  return ppocr_b200_roi_warp(src, src_step, src_rows, src_cols, d_m_invs,
                             d_crop_widths, d_dst_batch, batch, dst_h, dst_w,
                             output_bgr, PPOCR_B200_PREP_F32_NCHW, stream);
}

size_t ppocr_b200_db_components_workspace(int pages, int h, int w,
                                          int max_components) {
  if (pages <= 0 || h <= 0 || w <= 0 || max_components <= 0)
    return 0;
  return db_components_workspace(pages, h, w, max_components);
}

int ppocr_b200_db_components(const uint8_t *bitmap, const float *prob,
                             int pages, int h, int w, int max_components,
                             int *labels, int *counts, int *stats,
                             unsigned long long *prob_sum_q32, void *workspace,
                             cudaStream_t stream) {
  g_error.clear();
  if (pages < 0 || h < 0 || w < 0)
    return fail("invalid db components arguments");
  if (pages == 0 || h == 0 || w == 0)
    return 0;
  if (!bitmap || !labels || !counts || !stats || !prob_sum_q32 || !workspace ||
      max_components <= 0 ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) ||
      static_cast<long long>(pages) * h * w >= (1LL << 31))
    return fail("invalid db components arguments");
  return status(db_components(bitmap, prob, pages, h, w, max_components, labels,
                              counts, stats, prob_sum_q32, workspace, stream),
                "db components");
}

int ppocr_b200_device_free(void *p) {
  g_error.clear();
  return status(cudaFree(p), "cudaFree");
}

int ppocr_b200_f32_to_f16(const float *x, void *y, size_t valid, size_t total,
                          cudaStream_t stream) {
  g_error.clear();
  if (!x || !y || valid > total)
    return fail("invalid conversion arguments");
  return status(copy_input_f32(x, Hm(y), valid, total, stream), "f32_to_f16");
}

int ppocr_b200_f16_to_f32(const void *x, float *y, size_t n,
                          cudaStream_t stream) {
  g_error.clear();
  if (!x || !y)
    return fail("invalid conversion arguments");
  return status(half_to_float(H(x), y, n, stream), "f16_to_f32");
}

} // extern "C"
