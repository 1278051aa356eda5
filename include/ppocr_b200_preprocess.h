// Page and line preprocessing entry points of libppocr_b200.so: the
// detector's resize + normalize of a decoded page and the batched perspective
// ROI warp that cuts line crops out of it, on the device.
//
// Pages are u8 HWC, 3 channels, row pitch `step` bytes (the reference's
// GpuImage: native/include/ppocrv6_native/decode/gpu_image.h:7-16, passed
// here as data/step/rows/cols). Output either in the reference's layout
// (f32 NCHW planes, bit-identical to its kernels) or fused into the FP16
// NHWC tensor that ppocr_model_enqueue_nhwc_f16 takes, which removes the
// Model ABI's NCHW f32 input and its conversion pass from the page path.
// Return 0 on success, -1 on failure (message: ppocr_b200_last_error()).
#pragma once
#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Output layouts.
#define PPOCR_B200_PREP_F32_NCHW 0
#define PPOCR_B200_PREP_F16_NHWC 1

// Replaces kernels::cuda_resize_normalize_detector_padded
// (native/include/ppocrv6_native/kernels/detector_preprocess.h:10-13,
// native/src/kernels/detector_preprocess.cu:84-101): bilinear resize of the
// page into the upper-left content_h x content_w rectangle of a dst_h x dst_w
// canvas, white outside it, normalized (v/255 - mean)/std, channel order
// B, G, R. dst: [3][dst_h][dst_w] f32. Same argument checks and message
// ("invalid detector preprocess arguments") as the reference's exception.
int ppocr_b200_resize_normalize_detector_padded(
    const void *src, size_t src_step, int src_rows, int src_cols,
    float *dst_nchw, int dst_h, int dst_w, int content_h, int content_w,
    int source_is_bgr, cudaStream_t stream);
// Replaces kernels::cuda_resize_normalize_detector (detector_preprocess.h:
// 15-17, detector_preprocess.cu:77-82): the padded form with content = canvas.
int ppocr_b200_resize_normalize_detector(const void *src, size_t src_step,
                                         int src_rows, int src_cols,
                                         float *dst_nchw, int dst_h, int dst_w,
                                         int source_is_bgr, cudaStream_t stream);
// Extension: `images` equally sized pages (page i at src + i *
// src_image_bytes) in one launch, output layout `format`
// (PPOCR_B200_PREP_F16_NHWC: [images][dst_h][dst_w][3] fp16, the detector
// model's input; PPOCR_B200_PREP_F32_NCHW: [images][3][dst_h][dst_w] f32).
int ppocr_b200_detector_preprocess(const void *src, size_t src_step,
                                   int src_rows, int src_cols,
                                   size_t src_image_bytes, int images,
                                   void *dst, int dst_h, int dst_w,
                                   int content_h, int content_w,
                                   int source_is_bgr, int format,
                                   cudaStream_t stream);

// Replaces kernels::cuda_batch_roi_warp
// (native/include/ppocrv6_native/kernels/roi_warp.h:14-18,
// native/src/kernels/roi_warp.cu:113-131): crop b of `batch` samples the page
// through the inverse homography d_m_invs[9b..9b+8] (device, row-major 3x3)
// for x < d_crop_widths[b] (device), zero elsewhere; values v/127.5 - 1;
// output_bgr 1 swaps the first and last channel. dst: [batch][3][dst_h][dst_w]
// f32. batch <= 0 is a no-op, as in the reference.
int ppocr_b200_batch_roi_warp(const void *src, size_t src_step, int src_rows,
                              int src_cols, const float *d_m_invs,
                              const int *d_crop_widths, float *d_dst_batch,
                              int batch, int dst_h, int dst_w, int output_bgr,
                              cudaStream_t stream);
// Extension: the same warp written in layout `format` (FP16 NHWC
// [batch][dst_h][dst_w][3] feeds the recognizer's ppocr_model_enqueue_nhwc_f16
// directly).
int ppocr_b200_roi_warp(const void *src, size_t src_step, int src_rows,
                        int src_cols, const float *d_m_invs,
                        const int *d_crop_widths, void *dst, int batch,
                        int dst_h, int dst_w, int output_bgr, int format,
                        cudaStream_t stream);

// Line tensors for the recognizer (extension; replaces the server's CPU
// write_line_tensor, server/src/lines.rs:115-135 with server/src/main.rs:
// 1101-1150): `lines` decoded RGB images in one device buffer `pixels`
// (image i at byte offsets[i], widths[i] x heights[i], strides[i] bytes per
// row; the four arrays on the host) -> height 48, width ceil(48 * w / h),
// pixel-centre bilinear (an image already 48 high and of that width is
// copied), values (v/255 - 0.5)/0.5 when copied and v/127.5 - 1 when
// resampled, right-padded with 0 to `bucket` columns. `format`:
// PPOCR_B200_PREP_F16_NHWC [lines][48][bucket][3] fp16 (the recognizer's
// ppocr_model_enqueue_nhwc_f16 input) or PPOCR_B200_PREP_F32_NCHW
// [lines][3][48][bucket] f32 (the server's tensor). A line whose normalized
// width exceeds the bucket fails the call with the reference's message.
int ppocr_b200_line_tensors(const void *pixels, const long long *offsets,
                            const int *widths, const int *heights,
                            const int *strides, int lines, int bucket,
                            void *out, int format, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
