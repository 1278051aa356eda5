// B200 layer runtime: the operator API that generated `model.inc` graphs call.
//
// Same member names, method names, argument order and meaning as the
// reference's `struct Runtime` (native/src/compiled/runtime.cuh:377-1030), so
// a `model.inc` written by tools/compiled_models/export.py (or by hand in that
// style) compiles against this header unchanged:
//   t (tensor pointer table), ops (launch list), stream, weights, arena,
//   Scalar = half, conv / deconv / gemm_epilogue / matmul / layernorm /
//   softmax / binary / binary_fast / unary / transpose / slice / concat / pad /
//   pad_nhwc / pool / pool_nhwc / mean / mean_nhwc / resize_nearest /
//   resize_nearest_nhwc / run.
// Each method appends one closure to `ops` that launches a hand-written
// sm_100a kernel (kernels.h); there is no cuDNN/cuBLAS underneath and no CPU
// fallback. Unsupported operator forms throw std::runtime_error at build
// time, the way the reference throws for shapes it cannot serve.
//
// Extensions (not in the reference API): activation codes 3..6 on conv and
// gemm_epilogue (kernels.h / ptx.cuh), conv bias/activation for every conv
// kind (the reference honours them for depthwise only), deconv bias and
// activation, attention(), resize_nearest_add_nhwc(), upsample_concat_nhwc().
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <functional>
#include <memory>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#define CU(x)                                                                  \
  do {                                                                         \
    cudaError_t e_ = (x);                                                      \
    if (e_ != cudaSuccess)                                                     \
      throw std::runtime_error(std::string(#x) + ": " +                        \
                               cudaGetErrorString(e_));                        \
  } while (0)

using Scalar = half;
constexpr bool half_storage = true;
using Shape = std::vector<int>;
inline int count(const Shape &s) {
  return std::accumulate(s.begin(), s.end(), 1, std::multiplies<int>());
}

// Broadcast index helper used by generated fused_pointwise kernels
// (export.py broadcast_expression): constant divisor, then modulus
// (Modulus == 1: broadcast scalar; 0: no modulus).
template <int Divisor, int Modulus> __device__ __forceinline__ int flat_index(int i) {
  if constexpr (Modulus == 1)
    return 0;
  if constexpr (Divisor != 1)
    i /= Divisor;
  if constexpr (Modulus > 1)
    i %= Modulus;
  return i;
}

struct Runtime {
  cudaStream_t stream = nullptr;
  Scalar *weights = nullptr, *arena = nullptr;
  // Number of fp16 elements behind `weights`; lets matmul() recognise
  // constant right-hand sides. Set by the ABI shell before build_model.
  size_t weight_elements = 0;
  void *workspace = nullptr;
  size_t workspace_bytes = 0;
  static constexpr size_t workspace_limit = 1 << 20;
  std::vector<Scalar *> t;
  std::vector<std::function<void()>> ops;
  // One-time device work (weight re-layouts) run before the first run().
  std::vector<std::function<void()>> prepare;
  std::vector<std::string> op_names;

  Runtime();
  ~Runtime();
  Runtime(const Runtime &) = delete;
  Runtime &operator=(const Runtime &) = delete;

  void conv(int ai, int wi, int yi, Shape xs, Shape ws, Shape ys, Shape pad,
            Shape stride, Shape dilation, int groups,
            bool channels_last = false, bool input_channels_last = false,
            int bias_id = -1, int activation = 0);
  void deconv(int ai, int wi, int yi, Shape xs, Shape ws, Shape ys, Shape pad,
              Shape stride, Shape dilation, bool channels_last = false,
              int bias_id = -1, int activation = 0);
  void gemm_epilogue(int ai, int wi, int bi, int ri, int yi, int rows, int ci,
                     int co, int activation);
  void matmul(int a, int b, int y, int batches, int m, int n, int k);
  void layernorm(int a, int scale, int bias, int y, int rows, int cols,
                 float epsilon);
  void softmax(int a, int y, int rows, int cols);
  void binary(int a, int b, int y, Shape as, Shape bs, Shape ys, int op);
  template <int Op, int AD, int AM, int BD, int BM>
  void binary_fast(int a, int b, int y, int n) {
    binary_flat_op(a, b, y, n, AD, AM, BD, BM, Op);
  }
  void binary_flat_op(int a, int b, int y, int n, int ad, int am, int bd,
                      int bm, int op);
  void unary(int a, int y, int n, int op, float alpha, float beta);
  void transpose(int a, int y, Shape xs, Shape ys, Shape perm);
  void slice(int a, int y, Shape xs, Shape ys, Shape starts);
  void concat(int a, int b, int y, int rows, int na, int nb);
  void pad(int a, int y, Shape xs, Shape ys, int ph, int pw);
  void pad_nhwc(int a, int y, Shape xs, Shape ys, int ph, int pw);
  void pool(int a, int y, Shape xs, Shape ys, Shape k, Shape s, Shape p,
            bool maximum);
  void pool_nhwc(int a, int y, Shape xs, Shape ys, Shape k, Shape s, Shape p,
                 bool maximum);
  void mean(int a, int y, int rows, int cols);
  void mean_nhwc(int a, int y, int batch, int channels, int spatial);
  void resize_nearest(int a, int y, Shape xs, Shape ys, float sh, float sw);
  void resize_nearest_nhwc(int a, int y, Shape xs, Shape ys, float sh,
                           float sw);

  // ---- extensions
  // Fused multi-head self-attention over packed [lines][seq][3*heads*dh] rows.
  void attention(int qkv, int y, int lines, int seq, int heads, int head_dim,
                 float scale);
  // FPN step: y = nearest_resize(a) + addend (NHWC, logical NCHW shapes).
  void resize_nearest_add_nhwc(int a, int addend, int y, Shape xs, Shape ys,
                               float sh, float sw);
  // FPN tail: y = concat over channels of each source nearest-upsampled to
  // ys (scale = ys / xs per source), the resize_nearest_nhwc + concat chain
  // in one pass (NHWC, logical NCHW shapes, channels multiples of 8).
  void upsample_concat_nhwc(std::vector<int> srcs, int y, std::vector<Shape> xs, Shape ys);

  // Runs `prepare` once, then ops[first_op..] in order on `stream`.
  void run();
  // Declares that tensors `ids` are read after the ops recorded so far
  // (every method calls it for its inputs; the ABI shell calls it for the
  // model output). A depthwise conv fused into the 1x1 gemm_epilogue that
  // consumes it does not write its output; a later reader of that tensor
  // splits the fused op back into the two original launches.
  void reads(std::initializer_list<int> ids);
  bool prepared = false;
  // When the graph opens with the exporter's channels-last transpose of the
  // model input (t[0] NCHW -> t[input_nhwc_id] NHWC), the ABI shell writes
  // t[input_nhwc_id] directly and starts the launch list at first_op = 1.
  int input_nhwc_id = -1;
  int first_op = 0;

private:
  // The depthwise conv recorded by the last add(), if it can lead a fused
  // depthwise + pointwise block.
  struct PendingDw {
    int op = -1;
    int ai, wi, yi, bias_id, act, B, C, H, W, K;
  } last_dw_;
  // The tensor-core transposed conv recorded by the last add(), if it can
  // lead a fused DB tail (a 64 -> 1 transposed conv reading only its output).
  struct PendingDeconv {
    int op = -1;
    int ai, yi, B, H, W, Ci, Co, KH, KW, act;
    half *wp, *bp;
  } last_dc_;
  // The last gemm_epilogue without a residual, which an FPN resize-add of
  // its output can fold into (upsampled residual in the GEMM epilogue).
  struct PendingGemm {
    int op = -1;
    int ai, wi, bi, yi, rows, ci, co, act;
  } last_gemm_;
  // Fused pairs (depthwise + pointwise block, DB tail, lateral conv + FPN
  // resize-add) whose intermediate
  // tensor is not materialised; a later read of it splits the pair back.
  struct FusedDw {
    int op;
    int virt; // tensor id of the first op's output
    std::function<void()> dw_op, pw_op; // the first and second op, unfused
    const char *first_name = "depthwise", *second_name = "gemm_epilogue";
  };
  std::vector<FusedDw> fused_;
  std::vector<void *> owned_; // device buffers owned by this runtime
  void *own(size_t bytes);
  bool is_constant(const Scalar *p, size_t elements) const;
  void add(const char *name, std::function<void()> f);
  void add_fused_placeholder();
};
