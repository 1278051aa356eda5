// C entry points over the reference's own page preprocessing kernels
// (native/src/kernels/detector_preprocess.cu, native/src/kernels/roi_warp.cu),
// compiled unmodified where they lie into oracle/_ref/ by the Makefile
// beside this file. TEST INFRASTRUCTURE ONLY: run on the GPU box to pin the
// oracle's restatement and the B200 kernels against the reference itself.
#include "ppocrv6_native/kernels/detector_preprocess.h"
#include "ppocrv6_native/kernels/roi_warp.h"

extern "C" int ref_resize_normalize_detector_padded(
    void *src, size_t step, int rows, int cols, float *dst, int dst_h,
    int dst_w, int content_h, int content_w, int bgr, void *stream) {
  try {
    ppocrv6_native::GpuImage im{src, step, rows, cols};
    ppocrv6_native::kernels::cuda_resize_normalize_detector_padded(
        im, dst, dst_h, dst_w, content_h, content_w, bgr != 0,
        static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return -1;
  }
}

extern "C" int ref_batch_roi_warp(void *src, size_t step, int rows, int cols,
                                  const float *m_invs, const int *crop_widths,
                                  float *dst, int batch, int dst_h, int dst_w,
                                  int out_bgr, void *stream) {
  try {
    ppocrv6_native::GpuImage im{src, step, rows, cols};
    ppocrv6_native::kernels::cuda_batch_roi_warp(
        im, m_invs, crop_widths, dst, batch, dst_h, dst_w,
        out_bgr ? ppocrv6_native::kernels::ColorOrder::kBgr
                : ppocrv6_native::kernels::ColorOrder::kRgb,
        static_cast<cudaStream_t>(stream));
    return 0;
  } catch (...) {
    return -1;
  }
}
