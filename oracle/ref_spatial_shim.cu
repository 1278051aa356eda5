// C entry points over the reference's own NHWC depthwise and pooling kernels,
// compiled from native/src/compiled/spatial_kernels.cuh where it lies into
// oracle/_ref/ by the Makefile beside this file. TEST INFRASTRUCTURE ONLY:
// run on the GPU box to pin the oracle's depthwise restatement bit for bit.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
using Scalar = half;
#include "spatial_kernels.cuh"

template <int KH, int KW, int SH, int SW>
static int launch_dw(const half *x, const half *w, const half *bias, half *y,
                     int b, int c, int h, int wd, int oh, int ow, int ph,
                     int pw, int act, cudaStream_t s) {
  const int n = b * oh * ow * (c / 8);
  depthwise_nhwc_vec8<KH, KW, SH, 1, SW><<<(n + 127) / 128, 128, 0, s>>>(
      x, w, y, b, c, h, wd, oh, ow, ph, pw, bias, act);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

extern "C" int ref_depthwise_nhwc(const void *x, const void *w,
                                  const void *bias, void *y, int b, int c,
                                  int h, int wd, int oh, int ow, int kh,
                                  int kw, int sh, int sw, int ph, int pw,
                                  int act, void *stream) {
  auto X = static_cast<const half *>(x);
  auto Wt = static_cast<const half *>(w);
  auto B = static_cast<const half *>(bias);
  auto Y = static_cast<half *>(y);
  auto s = static_cast<cudaStream_t>(stream);
#define REF_DW(a, bb, c1, c2)                                                  \
  if (kh == a && kw == bb && sh == c1 && sw == c2)                             \
    return launch_dw<a, bb, c1, c2>(X, Wt, B, Y, b, c, h, wd, oh, ow, ph, pw,  \
                                    act, s);
  REF_DW(3, 3, 1, 1)
  REF_DW(3, 3, 2, 2)
  REF_DW(3, 3, 2, 1)
  REF_DW(5, 5, 1, 1)
  REF_DW(1, 7, 1, 1)
#undef REF_DW
  return -2;
}

extern "C" int ref_pool_nhwc(const void *x, void *y, int b, int c, int h,
                             int w, int oh, int ow, int kind, void *stream) {
  const int n = b * oh * ow * (c / 8);
  auto s = static_cast<cudaStream_t>(stream);
  if (kind == 0)
    pool_nhwc_vec8<2, 2, 1, 1, true><<<(n + 127) / 128, 128, 0, s>>>(
        static_cast<const half *>(x), static_cast<half *>(y), b, c, h, w, oh,
        ow, 0, 0);
  else
    pool_nhwc_vec8<3, 2, 3, 2, false><<<(n + 127) / 128, 128, 0, s>>>(
        static_cast<const half *>(x), static_cast<half *>(y), b, c, h, w, oh,
        ow, 0, 0);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
