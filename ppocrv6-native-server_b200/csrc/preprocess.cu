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
// operation order; the detector's division by the channel std is computed
// by a correction step proven to give the IEEE quotient for its operands),
// so the f32 output matches it bit for bit and the FP16 output is its
// round-to-nearest. Source bytes are gathered as aligned 32-bit words (a
// tap pair's six bytes in two or three loads instead of six byte loads) and
// converted to float on the FMA pipe.
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

// Exact u8 -> f32 on the FMA pipe: byte k of w placed in the low mantissa
// bits of 2^23 (one byte permute), minus 2^23.
__device__ __forceinline__ float byte_f(uint32_t w, uint32_t k) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | k)) - 8388608.0f;
}

// The two horizontally adjacent RGB pixels of a bilinear tap pair, bytes
// [o, o + 6) of a row (or [o, o + 3) when the pair is clamped to one pixel),
// fetched as the 1-3 aligned 32-bit words that hold them and funnel-shifted
// so lo = bytes o..o+3, hi = bytes o+4..o+7. Every word loaded holds at least
// one byte of the row, so no load leaves the page's memory.
struct Pair {
  uint32_t lo, hi;
};
__device__ __forceinline__ Pair load_pair(const uint8_t *p, bool two) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~static_cast<uintptr_t>(3));
  const uint32_t mis = static_cast<uint32_t>(a & 3);
  const uint32_t words = (mis + (two ? 6u : 3u) + 3u) >> 2;
  const uint32_t w0 = __ldg(w);
  const uint32_t w1 = words > 1 ? __ldg(w + 1) : 0u;
  const uint32_t w2 = words > 2 ? __ldg(w + 2) : 0u;
  Pair r;
  r.lo = __funnelshift_r(w0, w1, mis * 8);
  r.hi = __funnelshift_r(w1, w2, mis * 8);
  return r;
}
// Channel c (0..2) of the first / second pixel of a pair.
__device__ __forceinline__ float first_px(const Pair &q, int c) { return byte_f(q.lo, c); }
__device__ __forceinline__ float second_px(const Pair &q, int c, bool two) {
  if (!two)
    return byte_f(q.lo, c);
  return c == 0 ? byte_f(q.lo, 3) : byte_f(q.hi, c - 1);
}

// (v / 255 - mean) / std with the division as Markstein's correction step
// (P. Markstein, "IA-64 and Elementary Functions", 2000): q = a * (1/s),
// r = fma(-s, q, a) (exact), q' = fma(r, 1/s, q). With 1/s the correctly
// rounded reciprocal this equals the IEEE quotient a / s for the three
// divisors here and every |a| in [2^-103, 0.75] (checked exhaustively on the
// host, tests/test_cpu_preprocess_division.py); a = fma(v, 1/255, -mean)
// with v in [0, 255] is 0 or of magnitude in [2^-49, 0.6].
__device__ __forceinline__ float normalize(float v, float mean, float s, float inv_s) {
  const float a = __fmaf_rn(v, 1.0f / 255.0f, -mean);
  const float q = __fmul_rn(a, inv_s);
  const float r = __fmaf_rn(-s, q, a);
  return __fmaf_rn(r, inv_s, q);
}

// Both kernels work in three phases per thread: (1) the four pixels'
// sample coordinates and weights, (2) every source byte they need loaded
// (48 independent loads in flight: 4 pixels x 4 taps x 3 channels), (3) the
// interpolation and normalisation. Pixels that need no sample (padding,
// right of the crop, non-finite coordinates) load from offset 0 and are
// overwritten in phase 3.
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

  // phase 1
  int o0[kPix];
  bool two[kPix];
  float wx[kPix];
  bool in[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    const int x = x0 + p;
    in[p] = row_in && x < content_w;
    const float sx = (static_cast<float>(x) + 0.5f) * scale_x - 0.5f;
    const int x0u = static_cast<int>(floorf(sx));
    wx[p] = sx - static_cast<float>(x0u);
    const int a = min(max(x0u, 0), src_w - 1), b = min(max(x0u + 1, 0), src_w - 1);
    o0[p] = in[p] ? a * 3 : 0;
    two[p] = in[p] && b != a;
  }
  // phase 2
  Pair t[kPix], u[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    t[p] = load_pair(r0 + o0[p], two[p]);
    u[p] = load_pair(r1 + o0[p], two[p]);
  }
  // phase 3: per channel, top row blended in x, bottom row blended in x,
  // then the two blended in y (detector_preprocess.cu:12-33)
  constexpr float inv_std[3] = {1.0f / 0.229f, 1.0f / 0.224f, 1.0f / 0.225f};
  Rgb q[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int c = k == 0 ? ch0 : (k == 1 ? 1 : ch2);
      if (in[p]) {
        const float top = first_px(t[p], c) * (1.0f - wx[p]) + second_px(t[p], c, two[p]) * wx[p];
        const float bot = first_px(u[p], c) * (1.0f - wx[p]) + second_px(u[p], c, two[p]) * wx[p];
        const float v = top * (1.0f - wy) + bot * wy;
        q[p].c[k] = normalize(v, mean[k], stdv[k], inv_std[k]);
      } else {
        // the canvas colour: a constant expression, folded without fusion
        q[p].c[k] = (255.0f * inv255 - mean[k]) / stdv[k];
      }
    }
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
  const int bi = blockIdx.y;
  const int y = static_cast<int>(g / groups);
  const int x0 = static_cast<int>(g - static_cast<long long>(y) * groups) * kPix;
  const int n = min(kPix, dst_w - x0);
  // Every thread of the block reads the same nine coefficients: one
  // broadcast load each, no shared-memory round trip.
  float m[9];
#pragma unroll
  for (int k = 0; k < 9; ++k)
    m[k] = __ldg(m_invs + bi * 9 + k);
  const int crop_w = __ldg(crop_widths + bi);
  constexpr float inv127_5 = 1.0f / 127.5f;
  const float fy = static_cast<float>(y);

  // phase 1: inverse homography, clamps, weights and the taps' offsets
  long long ot[kPix], ou[kPix];
  bool two[kPix];
  float w[kPix][4];
  bool keep[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    const int x = x0 + p;
    const float fx = static_cast<float>(x);
    float den = m[6] * fx + m[7] * fy + m[8];
    if (fabsf(den) < 1e-7f)
      den = den < 0.0f ? -1e-7f : 1e-7f;
    const float inv = 1.0f / den;
    float sx = (m[0] * fx + m[1] * fy + m[2]) * inv;
    float sy = (m[3] * fx + m[4] * fy + m[5]) * inv;
    keep[p] = x < crop_w && isfinite(sx) && isfinite(sy);
    sx = keep[p] ? fminf(fmaxf(sx, -1.0f), static_cast<float>(src_w + 1)) : 0.0f;
    sy = keep[p] ? fminf(fmaxf(sy, -1.0f), static_cast<float>(src_h + 1)) : 0.0f;
    const int xi = static_cast<int>(floorf(sx));
    const int yi = static_cast<int>(floorf(sy));
    const float ax = sx - static_cast<float>(xi);
    const float ay = sy - static_cast<float>(yi);
    const int l = min(max(xi, 0), src_w - 1);
    const int rr = min(max(xi + 1, 0), src_w - 1);
    ot[p] = min(max(yi, 0), src_h - 1) * src_step + l * 3;
    ou[p] = min(max(yi + 1, 0), src_h - 1) * src_step + l * 3;
    two[p] = rr != l;
    w[p][0] = (1.0f - ax) * (1.0f - ay);
    w[p][1] = ax * (1.0f - ay);
    w[p][2] = (1.0f - ax) * ay;
    w[p][3] = ax * ay;
  }
  // phase 2
  Pair t[kPix], u[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    t[p] = load_pair(src + ot[p], two[p]);
    u[p] = load_pair(src + ou[p], two[p]);
  }
  // phase 3: Source channels are (R, G, B) in memory order for an RGB page;
  // the output keeps that order unless BGR is asked for.
  const int c0 = out_bgr ? 2 : 0, c2 = out_bgr ? 0 : 2;
  Rgb q[kPix];
#pragma unroll
  for (int p = 0; p < kPix; ++p) {
    float v[3];
#pragma unroll
    for (int c = 0; c < 3; ++c)
      v[c] = w[p][0] * first_px(t[p], c) + w[p][1] * second_px(t[p], c, two[p]) +
             w[p][2] * first_px(u[p], c) + w[p][3] * second_px(u[p], c, two[p]);
    q[p].c[0] = keep[p] ? v[c0] * inv127_5 - 1.0f : 0.0f;
    q[p].c[1] = keep[p] ? v[1] * inv127_5 - 1.0f : 0.0f;
    q[p].c[2] = keep[p] ? v[c2] * inv127_5 - 1.0f : 0.0f;
  }
  const long long plane = static_cast<long long>(dst_h) * dst_w;
  store4(q, x0, n, static_cast<long long>(y) * dst_w + x0, plane, bi, fmt, vec && n == kPix, dst);
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
