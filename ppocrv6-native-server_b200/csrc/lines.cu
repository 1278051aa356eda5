// Line-tensor construction on the device: decoded RGB line images of any
// size -> the recognizer's batch tensor, height 48, aspect kept, right-padded
// with the reference's 0.0 up to the bucket width.
//
// Reference: the server's write_line_tensor (server/src/lines.rs:115-135)
// with the shared RGB primitives write_rgb_tensor / write_resized_rgb_tensor
// (server/src/main.rs:1101-1150), run per line on the CPU:
//  * natural width ceil(48 * w / h) must fit the bucket (else the request
//    fails: "line normalized width N exceeds maximum B; split the line
//    crop", lines.rs:98-112);
//  * a 48-high line of exactly that width is copied: (v / 255 - 0.5) / 0.5;
//  * otherwise pixel-centre bilinear resize with source coordinates clamped
//    at 0 and the upper neighbour clamped to the last row/column:
//    value / 127.5 - 1;
//  * columns from the natural width to the bucket width are 0.
// Rust does not fuse multiplies into adds, so every operation here is a
// separately rounded IEEE operation (__fmul_rn & co.) in the reference's
// order: the f32 output is bit-identical, the FP16 NHWC output its
// round-to-nearest.
#include "kernels.h"

namespace pb2 {
namespace {

constexpr int kLineThreads = 256;

__device__ __forceinline__ float lerp_rs(float a, float b, float w) {
  // a * (1 - w) + b * w, each operation rounded
  return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, w)), __fmul_rn(b, w));
}

__global__ void __launch_bounds__(kLineThreads)
    line_tensor_kernel(const uint8_t *__restrict__ pixels, const __grid_constant__ LineBatch lb, void *__restrict__ out,
                       int bucket, int fmt) {
  const int line = blockIdx.y;
  const LineGeo geo = lb.line[line];
  const int i = blockIdx.x * kLineThreads + threadIdx.x;
  if (i >= 48 * bucket)
    return;
  const int y = i / bucket, x = i - y * bucket;
  float v[3] = {0.0f, 0.0f, 0.0f};
  if (x < geo.resized_width) {
    const uint8_t *img = pixels + geo.offset;
    if (geo.copy) {
      const uint8_t *p = img + static_cast<long long>(y) * geo.stride + x * 3;
#pragma unroll
      for (int c = 0; c < 3; ++c)
        v[c] = __fdiv_rn(__fsub_rn(__fdiv_rn(static_cast<float>(p[c]), 255.0f), 0.5f), 0.5f);
    } else {
      const float sx = fmaxf(__fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(x), 0.5f), geo.scale_x), 0.5f), 0.0f);
      const float sy = fmaxf(__fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(y), 0.5f), geo.scale_y), 0.5f), 0.0f);
      const int x0 = min(static_cast<int>(floorf(sx)), geo.width - 1), x1 = min(x0 + 1, geo.width - 1);
      const int y0 = min(static_cast<int>(floorf(sy)), geo.height - 1), y1 = min(y0 + 1, geo.height - 1);
      const float wx = __fsub_rn(sx, static_cast<float>(x0));
      const float wy = __fsub_rn(sy, static_cast<float>(y0));
      const uint8_t *r0 = img + static_cast<long long>(y0) * geo.stride;
      const uint8_t *r1 = img + static_cast<long long>(y1) * geo.stride;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float top = lerp_rs(static_cast<float>(r0[x0 * 3 + c]), static_cast<float>(r0[x1 * 3 + c]), wx);
        const float bot = lerp_rs(static_cast<float>(r1[x0 * 3 + c]), static_cast<float>(r1[x1 * 3 + c]), wx);
        v[c] = __fsub_rn(__fdiv_rn(lerp_rs(top, bot, wy), 127.5f), 1.0f);
      }
    }
  }
  if (fmt == PREP_F16_NHWC) {
    half *o = static_cast<half *>(out) + ((static_cast<long long>(line) * 48 + y) * bucket + x) * 3;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      o[c] = __float2half_rn(v[c]);
  } else {
    float *o = static_cast<float *>(out) + static_cast<long long>(line) * 3 * 48 * bucket + y * bucket + x;
#pragma unroll
    for (int c = 0; c < 3; ++c)
      o[static_cast<long long>(c) * 48 * bucket] = v[c];
  }
}

} // namespace

cudaError_t line_tensors(const uint8_t *pixels, const LineBatch &lb, int lines, void *out, int bucket, int fmt,
                         cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  if (lines > kMaxLineBatch || bucket <= 0)
    return cudaErrorInvalidValue;
  const dim3 grid((48 * bucket + kLineThreads - 1) / kLineThreads, lines);
  line_tensor_kernel<<<grid, kLineThreads, 0, s>>>(pixels, lb, out, bucket, fmt);
  return cudaGetLastError();
}

} // namespace pb2
