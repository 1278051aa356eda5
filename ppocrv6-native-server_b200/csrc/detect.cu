// DB detector tail: transposed convolution with kernel == stride (the DB
// head's 2x2 stride-2 upsampling) and the binarize step.
//
// Reference semantics (ppocrv6-native-server):
//   deconv    native/src/compiled/runtime.cuh:426-453 (cuDNN backward-data,
//             weights [Ci][KH][KW][Co] after the channels-last pass,
//             tools/compiled_models/export.py:590-600)
//   binarize  native/src/detection/db_postprocess.cpp:189-190
//             (cv::compare(pred, thresh, CMP_GT) -> 255 / 0)
#include "kernels.h"
#include "ptx.cuh"

namespace pb2 {
namespace {

// Thread = one output pixel x 8 output channels (Co % 8 == 0) or one output
// element (otherwise). With kernel == stride each output pixel has exactly
// one contributing input pixel and one filter tap.
__global__ void __launch_bounds__(256)
    deconv_kernel(const half *__restrict__ x, const half *__restrict__ w,
                  const half *__restrict__ bias, half *__restrict__ y,
                  long long total, int H, int W, int Ci, int Co, int KH,
                  int KW, int act, bool vec) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const int per = vec ? Co / 8 : Co;
  const int g = static_cast<int>(i % per);
  long long p = i / per;
  const int OW = W * KW, OH = H * KH;
  const int ox = static_cast<int>(p % OW);
  const int oy = static_cast<int>((p / OW) % OH);
  const long long n = p / (static_cast<long long>(OW) * OH);
  const int ix = ox / KW, dx = ox - ix * KW;
  const int iy = oy / KH, dy = oy - iy * KH;
  const half *px = x + ((n * H + iy) * W + ix) * Ci;
  const long long tap = static_cast<long long>(dy * KW + dx) * Co;
  const long long cstride = static_cast<long long>(KH) * KW * Co;
  if (vec) {
    const int co0 = g * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int ci = 0; ci < Ci; ++ci) {
      const float xv = __half2float(px[ci]);
      uint4 wv = __ldg(reinterpret_cast<const uint4 *>(w + ci * cstride + tap + co0));
      const half2 *wh = reinterpret_cast<const half2 *>(&wv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(wh[j]);
        acc[2 * j] = fmaf(xv, f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(xv, f.y, acc[2 * j + 1]);
      }
    }
    uint4 o;
    half2 *oh = reinterpret_cast<half2 *>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v0 = round_half(acc[2 * j]), v1 = round_half(acc[2 * j + 1]);
      if (bias) {
        v0 += __half2float(bias[co0 + 2 * j]);
        v1 += __half2float(bias[co0 + 2 * j + 1]);
      }
      oh[j] = __floats2half2_rn(apply_act(v0, act), apply_act(v1, act));
    }
    *reinterpret_cast<uint4 *>(y + p * Co + co0) = o;
  } else {
    float acc = 0.f;
    for (int ci = 0; ci < Ci; ++ci)
      acc = fmaf(__half2float(px[ci]), __half2float(w[ci * cstride + tap + g]),
                 acc);
    float v = round_half(acc);
    if (bias)
      v += __half2float(bias[g]);
    y[p * Co + g] = __float2half_rn(apply_act(v, act));
  }
}

// Few outputs per input pixel (KH*KW*Co <= NMAX, e.g. the DB head's last
// 64 -> 1 upsampling): thread = one input pixel computing all its taps'
// outputs, the input read once with 16-byte loads, the filter [Ci][taps*Co]
// in shared memory as fp32. Sums run over ci in order with fp32 FMAs.
template <int NMAX>
__global__ void __launch_bounds__(256)
    deconv_small_kernel(const half *__restrict__ x, const half *__restrict__ w,
                        const half *__restrict__ bias, half *__restrict__ y,
                        uint32_t pixels, FastDiv by_w, FastDiv by_h, int Ci,
                        int Co, int KH, int KW, int act) {
  pdl_begin();
  extern __shared__ float dsm[];
  const int nout = KH * KW * Co;
  for (int j = threadIdx.x; j < Ci * nout; j += blockDim.x)
    dsm[j] = __half2float(w[j]); // w is [Ci][KH][KW][Co] = [Ci][nout]
  __syncthreads();
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= pixels)
    return;
  const uint32_t r = by_w.div(p);
  const int iw = static_cast<int>(p - r * by_w.d);
  const uint32_t n = by_h.div(r);
  const int ih = static_cast<int>(r - n * by_h.d);
  const int W = static_cast<int>(by_w.d), H = static_cast<int>(by_h.d);
  float acc[NMAX];
#pragma unroll
  for (int o = 0; o < NMAX; ++o)
    acc[o] = 0.f;
  const half *px = x + static_cast<long long>(p) * Ci;
  if ((Ci & 7) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    for (int c8 = 0; c8 < Ci; c8 += 8) {
      uint4 v = __ldg(reinterpret_cast<const uint4 *>(px + c8));
      const half2 *h2 = reinterpret_cast<const half2 *>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 f = __half22float2(h2[j >> 1]);
        const float xv = (j & 1) ? f.y : f.x;
        const float *wr = dsm + (c8 + j) * nout;
#pragma unroll
        for (int o = 0; o < NMAX; ++o)
          if (o < nout)
            acc[o] = fmaf(xv, wr[o], acc[o]);
      }
    }
  } else {
    for (int ci = 0; ci < Ci; ++ci) {
      const float xv = __half2float(px[ci]);
#pragma unroll
      for (int o = 0; o < NMAX; ++o)
        if (o < nout)
          acc[o] = fmaf(xv, dsm[ci * nout + o], acc[o]);
    }
  }
  const long long OW = static_cast<long long>(W) * KW;
  const long long OH = static_cast<long long>(H) * KH;
#pragma unroll
  for (int o = 0; o < NMAX; ++o) {
    if (o >= nout)
      break;
    const int co = o % Co, tap = o / Co;
    const int a = tap / KW, b = tap - a * KW;
    float v = round_half(acc[o]);
    if (bias)
      v += __half2float(bias[co]);
    y[((static_cast<long long>(n) * OH + ih * KH + a) * OW + iw * KW + b) * Co + co] =
        __float2half_rn(apply_act(v, act));
  }
}

// Four or fewer outputs per input pixel with Ci = 8*G (the DB head's last
// 64 -> 1 upsampling): G threads share an input pixel, each loading one
// 16-byte group of 8 channels (a warp reads 32/G pixels = 512 contiguous
// bytes per load) and holding that group's filter rows in registers. A warp
// issues the loads of U such pixel sets before any arithmetic. The four
// partial sums are reduce-scattered across the G lanes (two halving
// exchanges, then a plain butterfly: the same pairwise sums as a full
// butterfly of every output), leaving output o on the lanes whose group
// bits (G/2, G/4) spell o; the lowest of those lanes stores it.
// Grid-stride over pixels.
template <int G, int U>
__global__ void __launch_bounds__(256)
    deconv_group_kernel(const half *__restrict__ x, const half *__restrict__ w,
                        const half *__restrict__ bias, half *__restrict__ y,
                        uint32_t pixels, FastDiv by_w, FastDiv by_h, int Co,
                        int KH, int KW, int act) {
  pdl_begin();
  constexpr int NOUT = 4;
  constexpr uint32_t PPW = 32 / G; // pixels per warp per load
  const int nout = KH * KW * Co;
  const int lane = threadIdx.x & 31, g = lane % G;
  float wr[8][NOUT]; // this group's 8 channels x outputs
#pragma unroll
  for (int c = 0; c < 8; ++c)
#pragma unroll
    for (int o = 0; o < NOUT; ++o)
      wr[c][o] = o < nout ? __half2float(w[(g * 8 + c) * nout + o]) : 0.f;
  const bool hi1 = (g & (G / 2)) != 0, hi2 = (g & (G / 4)) != 0;
  const int mine = (hi1 ? 2 : 0) + (hi2 ? 1 : 0); // the output this lane ends with
  const bool writer = (g & (G / 4 - 1)) == 0 && mine < nout;
  const int co = mine % Co, tap = mine / Co;
  const int ta = tap / KW, tb = tap - ta * KW;
  const float bv = bias && mine < nout ? __half2float(bias[co]) : 0.f;
  const int W = static_cast<int>(by_w.d), H = static_cast<int>(by_h.d);
  const long long OW = static_cast<long long>(W) * KW;
  const long long OH = static_cast<long long>(H) * KH;
  const uint32_t warps = gridDim.x * (blockDim.x / 32);
  const uint32_t step = warps * PPW * U;
  // The loop bound is uniform across a warp, so every lane reaches the
  // shuffles; lanes past the last pixel compute zeros and store nothing.
  for (uint32_t pw = (blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5)) * PPW * U; pw < pixels;
       pw += step) {
    uint4 u[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const uint32_t p = pw + k * PPW + lane / G;
      u[k] = p < pixels ? __ldcs(reinterpret_cast<const uint4 *>(x + static_cast<long long>(p) * G * 8) + g)
                        : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const uint32_t p = pw + k * PPW + lane / G;
      const half2 *h2 = reinterpret_cast<const half2 *>(&u[k]);
      // Outputs (0, 1) and (2, 3) as two packed fp32 chains: each lane of
      // fma.rn.f32x2 rounds like fmaf, so the sums are the scalar ones.
      float2 a01 = make_float2(0.f, 0.f), a23 = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        ffma2(a01, make_float2(f.x, f.x), make_float2(wr[2 * j][0], wr[2 * j][1]));
        ffma2(a23, make_float2(f.x, f.x), make_float2(wr[2 * j][2], wr[2 * j][3]));
        ffma2(a01, make_float2(f.y, f.y), make_float2(wr[2 * j + 1][0], wr[2 * j + 1][1]));
        ffma2(a23, make_float2(f.y, f.y), make_float2(wr[2 * j + 1][2], wr[2 * j + 1][3]));
      }
      const float acc[NOUT] = {a01.x, a01.y, a23.x, a23.y};
      // Reduce-scatter: keep {0,1} or {2,3}, then one of the pair.
      const float s0 = __shfl_xor_sync(0xffffffffu, hi1 ? acc[0] : acc[2], G / 2);
      const float s1 = __shfl_xor_sync(0xffffffffu, hi1 ? acc[1] : acc[3], G / 2);
      const float k0 = (hi1 ? acc[2] : acc[0]) + s0;
      const float k1 = (hi1 ? acc[3] : acc[1]) + s1;
      float v = (hi2 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, hi2 ? k0 : k1, G / 4);
#pragma unroll
      for (int off = G / 8; off; off >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, off);
      if (writer && p < pixels) {
        const uint32_t r = by_w.div(p);
        const int iw = static_cast<int>(p - r * by_w.d);
        const uint32_t n = by_h.div(r);
        const int ih = static_cast<int>(r - n * by_h.d);
        float o = round_half(v);
        if (bias)
          o += bv;
        y[((static_cast<long long>(n) * OH + ih * KH + ta) * OW + iw * KW + tb) * Co + co] =
            __float2half_rn(apply_act(o, act));
      }
    }
  }
}

// Four float4 loads in flight per thread (16 probabilities), 4-byte stores.
__global__ void __launch_bounds__(256)
    binarize_kernel(const float *__restrict__ prob, uint8_t *__restrict__ map,
                    size_t n, float thresh) {
  pdl_begin();
  const size_t nv = n / 4; // whole float4 vectors
  const size_t v0 = static_cast<size_t>(blockIdx.x) * blockDim.x * 4 + threadIdx.x;
  float4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const size_t i = v0 + static_cast<size_t>(k) * blockDim.x;
    if (i < nv)
      v[k] = __ldcs(reinterpret_cast<const float4 *>(prob) + i);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const size_t i = v0 + static_cast<size_t>(k) * blockDim.x;
    if (i < nv) {
      uchar4 o;
      o.x = v[k].x > thresh ? 255 : 0;
      o.y = v[k].y > thresh ? 255 : 0;
      o.z = v[k].z > thresh ? 255 : 0;
      o.w = v[k].w > thresh ? 255 : 0;
      reinterpret_cast<uchar4 *>(map)[i] = o;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < n - nv * 4) {
    const size_t i = nv * 4 + threadIdx.x;
    map[i] = prob[i] > thresh ? 255 : 0;
  }
}

} // namespace

cudaError_t binarize(const float *prob, uint8_t *map, size_t n, float thresh,
                     cudaStream_t s) {
  if (!n)
    return cudaSuccess;
  if ((reinterpret_cast<uintptr_t>(prob) & 15) ||
      (reinterpret_cast<uintptr_t>(map) & 3))
    return cudaErrorInvalidValue;
  const size_t vectors = n / 4;
  const size_t blocks = vectors ? (vectors + 1023) / 1024 : 1;
  launch_pdl(binarize_kernel, static_cast<unsigned>(blocks), 256, 0, s, prob, map, n, thresh);
  return cudaGetLastError();
}

cudaError_t deconv_pack(const half *w, const half *bias, half *wpacked,
                        half *bias_rep, int Ci, int Co, int KH, int KW,
                        cudaStream_t s) {
  const int N = KH * KW * Co;
  cudaError_t e = transpose2d(w, wpacked, 1, Ci, N, s);
  if (e != cudaSuccess || !bias || !bias_rep)
    return e;
  for (int t = 0; t < KH * KW; ++t) {
    e = cudaMemcpyAsync(bias_rep + static_cast<size_t>(t) * Co, bias,
                        sizeof(half) * Co, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

cudaError_t deconv_kxk(const half *x, const half *w, const half *bias, half *y,
                       int batch, int H, int W, int Ci, int Co, int KH, int KW,
                       int act, cudaStream_t s) {
  if (batch <= 0)
    return cudaSuccess;
  const long long pixels = static_cast<long long>(batch) * H * W;
  const int nout = KH * KW * Co;
  if (nout <= 4 && (Ci == 64 || Ci == 128 || Ci == 256) && pixels < (1LL << 31) &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const int G = Ci / 8; // threads per pixel
    constexpr int U = 4;   // pixel sets loaded per warp before arithmetic
    const long long per_block = 256 / G * U;
    long long blocks = (pixels + per_block - 1) / per_block;
    const long long cap = static_cast<long long>(sm_count()) * 8;
    if (blocks > cap)
      blocks = cap;
    auto k = G == 8 ? deconv_group_kernel<8, U> : G == 16 ? deconv_group_kernel<16, U>
                                                          : deconv_group_kernel<32, U>;
    launch_pdl(k, static_cast<unsigned>(blocks), 256, 0, s, x, w, bias, y,
        static_cast<uint32_t>(pixels), FastDiv(W), FastDiv(H), Co, KH, KW, act);
    return cudaGetLastError();
  }
  const size_t smem = sizeof(float) * static_cast<size_t>(Ci) * nout;
  if (nout <= 16 && pixels < (1LL << 31) && smem <= 48 * 1024) {
    const unsigned blocks = static_cast<unsigned>((pixels + 255) / 256);
    if (nout <= 4)
      launch_pdl(deconv_small_kernel<4>, blocks, 256, smem, s, x, w, bias, y,
          static_cast<uint32_t>(pixels), FastDiv(W), FastDiv(H), Ci, Co, KH, KW, act);
    else
      launch_pdl(deconv_small_kernel<16>, blocks, 256, smem, s, x, w, bias, y,
          static_cast<uint32_t>(pixels), FastDiv(W), FastDiv(H), Ci, Co, KH, KW, act);
    return cudaGetLastError();
  }
  const bool vec = Co % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  const long long total = static_cast<long long>(batch) * H * KH * W * KW *
                          (vec ? Co / 8 : Co);
  launch_pdl(deconv_kernel, static_cast<unsigned>((total + 255) / 256), 256, 0, s, x, w, bias, y,
      total, H, W, Ci, Co, KH, KW, act, vec);
  return cudaGetLastError();
}

} // namespace pb2
