// Page and line preprocessing on the device: the detector's resize +
// normalize of a decoded u8 page and the batched perspective ROI warp that
// cuts the recognizer's line crops out of it.
//
// Reference semantics (ppocrv6-native-server):
//   detector  native/src/kernels/detector_preprocess.cu:12-73, 84-101
//             (pixel-centre bilinear resize of the content rectangle, edge
//             clamp, white (255) outside it, (v/255 - mean)/std per channel,
//             output channel order B, G, R with means .485/.456/.406 and
//             stds .229/.224/.225, f32 NCHW)
//   roi warp  native/src/kernels/roi_warp.cu:10-131 (inverse homography per
//             crop, denominator clamped to +-1e-7, source coordinates
//             clamped to [-1, size + 1], clamped-edge bilinear, v/127.5 - 1,
//             zeros right of the crop width and for non-finite coordinates)
// Caller: native/src/full_page/full_page_worker.cpp:345-349, 467-471.
//
// The B200 form writes either the reference's f32 NCHW planes or, fused,
// the FP16 NHWC tensor the compiled models take (the Model ABI's NCHW f32
// input and its conversion pass then disappear from the page path). Each
// thread makes four horizontally adjacent pixels so every store is a whole
// 8-byte (FP16 NHWC: 12 halves = 3 x 8 B) or 16-byte (f32 plane) vector.
// The arithmetic is the reference's expression for expression (same
// operation order, IEEE division), so the f32 output matches it bit for bit
// and the FP16 output is its round-to-nearest.
#include "kernels.h"

namespace pb2 {
namespace {

constexpr int kPrepThreads = 256;
constexpr int kPix = 4; // output pixels per thread

struct Rgb {
  float c[3];
};

// Stores four pixels' three channels (q[pixel].c[channel], already in the
// output channel order) at pixel x0 of output row `row` (row-major pixel
// index of the first pixel) of image `img`.
__device__ __forceinline__ void store4(const Rgb (&q)[kPix], int x0, int n,
                                       long long pix0, long long plane,
                                       long long img, int fmt, bool vec,
                                       void *dst) {
  if (fmt == PREP_F16_NHWC) {
    half *o = static_cast<half *>(dst) + (img * plane + pix0) * 3;
    if (vec) {
      half h[12];
#pragma unroll
      for (int p = 0; p < kPix; ++p)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          h[p * 3 + c] = __float2half_rn(q[p].c[c]);
      uint2 *o2 = reinterpret_cast<uint2 *>(o);
      const uint2 *h2 = reinterpret_cast<const uint2 *>(h);
      o2[0] = h2[0];
      o2[1] = h2[1];
      o2[2] = h2[2];
    } else {
      for (int p = 0; p < n; ++p)
        for (int c = 0; c < 3; ++c)
          o[p * 3 + c] = __float2half_rn(q[p].c[c]);
    }
  } else {
    float *o = static_cast<float *>(dst) + img * 3 * plane + pix0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float *oc = o + c * plane;
      if (vec) {
        *reinterpret_cast<float4 *>(oc) = make_float4(q[0].c[c], q[1].c[c], q[2].c[c], q[3].c[c]);
      } else {
        for (int p = 0; p < n; ++p)
          oc[p] = q[p].c[c];
      }
    }
  }
  (void)x0;
}

// One channel of a clamped-edge bilinear sample: top row blended in x, bottom
// row blended in x, then the two blended in y (detector_preprocess.cu:12-33).
__device__ __forceinline__ float bilerp_xy(const uint8_t *r0, const uint8_t *r1, int o0,
                                           int o1, float wx, float wy, int c) {
  const float top = static_cast<float>(r0[o0 + c]) * (1.0f - wx) + static_cast<float>(r0[o1 + c]) * wx;
  const float bot = static_cast<float>(r1[o0 + c]) * (1.0f - wx) + static_cast<float>(r1[o1 + c]) * wx;
  return top * (1.0f - wy) + bot * wy;
}

__global__ void __launch_bounds__(kPrepThreads)
    detector_prep_kernel(const uint8_t *__restrict__ src, int src_h, int src_w,
                         long long src_step, long long src_image_bytes,
                         void *__restrict__ dst, int dst_h, int dst_w,
                         int content_h, int content_w, int bgr, int fmt,
                         bool vec) {
  const int groups = (dst_w + kPix - 1) / kPix;
  const long long g = static_cast<long long>(blockIdx.x) * kPrepThreads + threadIdx.x;
  if (g >= static_cast<long long>(groups) * dst_h)
    return;
  const int img = blockIdx.y;
  const int y = static_cast<int>(g / groups);
  const int x0 = static_cast<int>(g - static_cast<long long>(y) * groups) * kPix;
  const int n = min(kPix, dst_w - x0);
  const uint8_t *im = src + img * src_image_bytes;

  const float scale_x = static_cast<float>(src_w) / static_cast<float>(content_w);
  const float scale_y = static_cast<float>(src_h) / static_cast<float>(content_h);
  // Output channel k reads source channel ch[k] (B, G, R order out).
  const int ch0 = bgr ? 0 : 2, ch2 = bgr ? 2 : 0;
  constexpr float inv255 = 1.0f / 255.0f;
  constexpr float mean[3] = {0.485f, 0.456f, 0.406f};
  constexpr float stdv[3] = {0.229f, 0.224f, 0.225f};

  // Row geometry is shared by the four pixels.
  const float sy = (static_cast<float>(y) + 0.5f) * scale_y - 0.5f;
  const int y0u = static_cast<int>(floorf(sy));
  const float wy = sy - static_cast<float>(y0u);
  const uint8_t *r0 = im + min(max(y0u, 0), src_h - 1) * src_step;
  const uint8_t *r1 = im + min(max(y0u + 1, 0), src_h - 1) * src_step;
  const bool row_in = y < content_h;

  Rgb q[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    const int x = x0 + p;
    float v[3];
    if (!row_in || x >= content_w) {
      v[0] = v[1] = v[2] = 255.0f;
    } else {
      const float sx = (static_cast<float>(x) + 0.5f) * scale_x - 0.5f;
      const int x0u = static_cast<int>(floorf(sx));
      const float wx = sx - static_cast<float>(x0u);
      const int o0 = min(max(x0u, 0), src_w - 1) * 3;
      const int o1 = min(max(x0u + 1, 0), src_w - 1) * 3;
      v[0] = bilerp_xy(r0, r1, o0, o1, wx, wy, ch0);
      v[1] = bilerp_xy(r0, r1, o0, o1, wx, wy, 1);
      v[2] = bilerp_xy(r0, r1, o0, o1, wx, wy, ch2);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c)
      q[p].c[c] = (v[c] * inv255 - mean[c]) / stdv[c];
  }
  const long long plane = static_cast<long long>(dst_h) * dst_w;
  store4(q, x0, n, static_cast<long long>(y) * dst_w + x0, plane, img, fmt, vec && n == kPix, dst);
}

__global__ void __launch_bounds__(kPrepThreads)
    roi_warp_kernel(const uint8_t *__restrict__ src, int src_h, int src_w,
                    long long src_step, const float *__restrict__ m_invs,
                    const int *__restrict__ crop_widths, void *__restrict__ dst,
                    int dst_h, int dst_w, int out_bgr, int fmt, bool vec) {
  const int groups = (dst_w + kPix - 1) / kPix;
  const long long g = static_cast<long long>(blockIdx.x) * kPrepThreads + threadIdx.x;
  if (g >= static_cast<long long>(groups) * dst_h)
    return;
  const int b = blockIdx.y;
  const int y = static_cast<int>(g / groups);
  const int x0 = static_cast<int>(g - static_cast<long long>(y) * groups) * kPix;
  const int n = min(kPix, dst_w - x0);
  // Every thread of the block reads the same nine coefficients: one
  // broadcast load each, no shared-memory round trip.
  float m[9];
#pragma unroll
  for (int k = 0; k < 9; ++k)
    m[k] = __ldg(m_invs + b * 9 + k);
  const int crop_w = __ldg(crop_widths + b);
  constexpr float inv127_5 = 1.0f / 127.5f;
  const float fy = static_cast<float>(y);

  Rgb q[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    const int x = x0 + p;
    q[p].c[0] = q[p].c[1] = q[p].c[2] = 0.0f;
    if (x >= crop_w)
      continue;
    const float fx = static_cast<float>(x);
    float den = m[6] * fx + m[7] * fy + m[8];
    if (fabsf(den) < 1e-7f)
      den = den < 0.0f ? -1e-7f : 1e-7f;
    const float inv = 1.0f / den;
    float sx = (m[0] * fx + m[1] * fy + m[2]) * inv;
    float sy = (m[3] * fx + m[4] * fy + m[5]) * inv;
    if (!isfinite(sx) || !isfinite(sy))
      continue;
    sx = fminf(fmaxf(sx, -1.0f), static_cast<float>(src_w + 1));
    sy = fminf(fmaxf(sy, -1.0f), static_cast<float>(src_h + 1));
    const int xi = static_cast<int>(floorf(sx));
    const int yi = static_cast<int>(floorf(sy));
    const float ax = sx - static_cast<float>(xi);
    const float ay = sy - static_cast<float>(yi);
    const uint8_t *t = src + min(max(yi, 0), src_h - 1) * src_step;
    const uint8_t *u = src + min(max(yi + 1, 0), src_h - 1) * src_step;
    const int l = min(max(xi, 0), src_w - 1) * 3;
    const int rr = min(max(xi + 1, 0), src_w - 1) * 3;
    const float w00 = (1.0f - ax) * (1.0f - ay);
    const float w10 = ax * (1.0f - ay);
    const float w01 = (1.0f - ax) * ay;
    const float w11 = ax * ay;
    float v[3];
#pragma unroll
    for (int c = 0; c < 3; ++c)
      v[c] = w00 * static_cast<float>(__ldg(t + l + c)) + w10 * static_cast<float>(__ldg(t + rr + c)) +
             w01 * static_cast<float>(__ldg(u + l + c)) + w11 * static_cast<float>(__ldg(u + rr + c));
    // Source channels are (R, G, B) in memory order for an RGB page; the
    // output keeps that order unless BGR is asked for.
    const int c0 = out_bgr ? 2 : 0, c2 = out_bgr ? 0 : 2;
    q[p].c[0] = v[c0] * inv127_5 - 1.0f;
    q[p].c[1] = v[1] * inv127_5 - 1.0f;
    q[p].c[2] = v[c2] * inv127_5 - 1.0f;
  }
  const long long plane = static_cast<long long>(dst_h) * dst_w;
  store4(q, x0, n, static_cast<long long>(y) * dst_w + x0, plane, b, fmt, vec && n == kPix, dst);
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

} // namespace

cudaError_t detector_preprocess(const uint8_t *src, int src_h, int src_w,
                                long long src_step, long long src_image_bytes,
                                int images, void *dst, int dst_h, int dst_w,
                                int content_h, int content_w, int source_is_bgr,
                                int fmt, cudaStream_t s) {
  if (images <= 0)
    return cudaSuccess;
  const int groups = (dst_w + kPix - 1) / kPix;
  const long long items = static_cast<long long>(groups) * dst_h;
  const long long blocks = (items + kPrepThreads - 1) / kPrepThreads;
  if (blocks > 0x7fffffffLL || images > 65535)
    return cudaErrorInvalidValue;
  // Whole-vector stores need every row to start on a vector boundary.
  const bool vec = dst_w % kPix == 0 && aligned(dst, 16);
  detector_prep_kernel<<<dim3(static_cast<unsigned>(blocks), images), kPrepThreads, 0, s>>>(
      src, src_h, src_w, src_step, src_image_bytes, dst, dst_h, dst_w, content_h, content_w,
      source_is_bgr, fmt, vec);
  return cudaGetLastError();
}

cudaError_t roi_warp(const uint8_t *src, int src_h, int src_w, long long src_step,
                     const float *m_invs, const int *crop_widths, void *dst,
                     int batch, int dst_h, int dst_w, int out_bgr, int fmt,
                     cudaStream_t s) {
  if (batch <= 0 || dst_h <= 0 || dst_w <= 0)
    return cudaSuccess;
  const int groups = (dst_w + kPix - 1) / kPix;
  const long long items = static_cast<long long>(groups) * dst_h;
  const long long blocks = (items + kPrepThreads - 1) / kPrepThreads;
  if (blocks > 0x7fffffffLL || batch > 65535)
    return cudaErrorInvalidValue;
  const bool vec = dst_w % kPix == 0 && aligned(dst, 16);
  roi_warp_kernel<<<dim3(static_cast<unsigned>(blocks), batch), kPrepThreads, 0, s>>>(
      src, src_h, src_w, src_step, m_invs, crop_widths, dst, dst_h, dst_w, out_bgr, fmt, vec);
  return cudaGetLastError();
}

} // namespace pb2
