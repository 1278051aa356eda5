// Memory-bound NHWC kernels of the layer path: depthwise convolution with the
// fused bias/activation epilogue, small-Ci direct convolution (stem), pooling,
// padding, nearest resize (+ fused FPN add), row concat, transposes, gathers,
// broadcast elementwise ops and the ABI input/output conversions.
//
// Reference semantics followed (file:line in ppocrv6-native-server):
//   depthwise    native/src/compiled/spatial_kernels.cuh:31-109 (tap order,
//                fp16 rounding of the sum before bias, activation after)
//   pool         spatial_kernels.cuh:156-193, 289-308 (count excludes pad)
//   pad          spatial_kernels.cuh:9-22, 225-236
//   resize       native/src/compiled/runtime.cuh:356-376 (asymmetric, floor)
//   concat       runtime.cuh:145-160
//   transpose    runtime.cuh:125-144, gather/slice 125-129
//   binary/unary runtime.cuh:73-124
//   copy_input   native/src/compiled/model_library.cu:15-25
// All kernels move 16-byte vectors (8 fp16 channels) where the layout allows.
#include "kernels.h"
#include "ptx.cuh"

namespace pb2 {
namespace {

constexpr int kBlock = 256;

union Pack8 {
  uint4 u;
  half2 h[4];
};

inline unsigned blocks_for(long long n, int per_block = kBlock) {
  long long b = (n + per_block - 1) / per_block;
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

// ------------------------------------------------------------- depthwise
// Work item = 8 channels x PIX consecutive output columns of one output row;
// consecutive threads take consecutive channel groups of the same pixels, so
// every 16-byte load and store is coalesced across the warp. Per filter row
// the item loads its input strip ((PIX-1)*SW + KW pixels) once into
// registers. The filter is staged in shared memory tap-major ([tap][C]) so a
// tap's 8 weights are one 16-byte load. Blocks loop over items (grid sized
// to the SM count) so the filter is staged once per block. Sums follow the
// reference's tap order (row a, then column b) with fp32 FMAs.
template <int KH, int KW, int SH, int SW, int PIX, int ACT>
__global__ void __launch_bounds__(kBlock, 4)
    depthwise_kernel(const half *__restrict__ x, const half *__restrict__ w,
                     const half *__restrict__ bias, half *__restrict__ y,
                     int batch, int C, int H, int W, int OH, int OW, int PH,
                     int PW, int act, uint32_t total, FastDiv by_groups,
                     FastDiv by_tiles, FastDiv by_oh) {
  pdl_begin();
  extern __shared__ uint4 dw_smem[];
  half *ws = reinterpret_cast<half *>(dw_smem);
  constexpr int TAPS = KH * KW;
  for (int j = threadIdx.x; j < C * TAPS; j += blockDim.x) {
    const int c = j / TAPS, tap = j - c * TAPS; // w is [C][KH][KW]
    ws[tap * C + c] = w[j];
  }
  __syncthreads();
  constexpr int NCOL = (PIX - 1) * SW + KW;
  // Item i = ((n * OH + oh) * tiles + tile) * groups + g, below 2^31.
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += gridDim.x * blockDim.x) {
    const uint32_t t0 = by_groups.div(i);
    const int g = static_cast<int>(i - t0 * by_groups.d);
    const uint32_t t1 = by_tiles.div(t0);
    const int tile = static_cast<int>(t0 - t1 * by_tiles.d);
    const uint32_t n_ = by_oh.div(t1);
    const int oh = static_cast<int>(t1 - n_ * by_oh.d);
    const int n = static_cast<int>(n_);
    const int c0 = g * 8;
    const int ow0 = tile * PIX;
    const int col0 = ow0 * SW - PW;

    float acc[PIX][8];
#pragma unroll
    for (int p = 0; p < PIX; ++p)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        acc[p][j] = 0.f;

    const half *xn = x + static_cast<long long>(n) * H * W * C + c0;
#pragma unroll
    for (int a = 0; a < KH; ++a) {
      const int r = oh * SH - PH + a;
      if (r < 0 || r >= H)
        continue;
      Pack8 strip[NCOL];
#pragma unroll
      for (int k = 0; k < NCOL; ++k) {
        const int c = col0 + k;
        strip[k].u = (c >= 0 && c < W)
                         ? __ldg(reinterpret_cast<const uint4 *>(
                               xn + (static_cast<long long>(r) * W + c) * C))
                         : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int b = 0; b < KW; ++b) {
        const uint4 wt = *reinterpret_cast<const uint4 *>(ws + (a * KW + b) * C + c0);
#pragma unroll
        for (int p = 0; p < PIX; ++p) {
          // fp16 x fp16 + fp32 in one instruction: same bits as fmaf on the
          // converted values.
          const uint4 xv = strip[p * SW + b].u;
          fma2_h(acc[p][0], acc[p][1], xv.x, wt.x);
          fma2_h(acc[p][2], acc[p][3], xv.y, wt.y);
          fma2_h(acc[p][4], acc[p][5], xv.z, wt.z);
          fma2_h(acc[p][6], acc[p][7], xv.w, wt.w);
        }
      }
    }
    float bv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      bv[j] = bias ? __half2float(bias[c0 + j]) : 0.f;
#pragma unroll
    for (int p = 0; p < PIX; ++p) {
      const int ow = ow0 + p;
      if (ow >= OW)
        break;
      Pack8 o;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v0 = round_half(acc[p][2 * j]);
        float v1 = round_half(acc[p][2 * j + 1]);
        if (bias) {
          v0 = act_t<ACT>(v0 + bv[2 * j], act);
          v1 = act_t<ACT>(v1 + bv[2 * j + 1], act);
        }
        o.h[j] = __floats2half2_rn(v0, v1);
      }
      *reinterpret_cast<uint4 *>(
          y + ((static_cast<long long>(n) * OH + oh) * OW + ow) * C + c0) =
          o.u;
    }
  }
}

// Any filter size / stride: same structure, runtime loop bounds.
__global__ void __launch_bounds__(kBlock)
    depthwise_generic_kernel(const half *__restrict__ x,
                             const half *__restrict__ w,
                             const half *__restrict__ bias,
                             half *__restrict__ y, int batch, int C, int H,
                             int W, int OH, int OW, int KH, int KW, int SH,
                             int SW, int PH, int PW, int act) {
  pdl_begin();
  const int groups = C >> 3;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(batch) * OH * OW * groups;
  if (i >= total)
    return;
  const int g = static_cast<int>(i % groups);
  long long t = i / groups;
  const int ow = static_cast<int>(t % OW);
  t /= OW;
  const int oh = static_cast<int>(t % OH);
  const int n = static_cast<int>(t / OH);
  const int c0 = g * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const half *xn = x + static_cast<long long>(n) * H * W * C;
  for (int a = 0; a < KH; ++a) {
    const int r = oh * SH - PH + a;
    if (r < 0 || r >= H)
      continue;
    for (int b = 0; b < KW; ++b) {
      const int c = ow * SW - PW + b;
      if (c < 0 || c >= W)
        continue;
      Pack8 v;
      v.u = __ldg(reinterpret_cast<const uint4 *>(
          xn + (static_cast<long long>(r) * W + c) * C + c0));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(v.h[j]);
        acc[2 * j] = fmaf(
            f.x, __half2float(w[(c0 + 2 * j) * (KH * KW) + a * KW + b]),
            acc[2 * j]);
        acc[2 * j + 1] = fmaf(
            f.y, __half2float(w[(c0 + 2 * j + 1) * (KH * KW) + a * KW + b]),
            acc[2 * j + 1]);
      }
    }
  }
  Pack8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v0 = round_half(acc[2 * j]);
    float v1 = round_half(acc[2 * j + 1]);
    if (bias) {
      v0 = apply_act(v0 + __half2float(bias[c0 + 2 * j]), act);
      v1 = apply_act(v1 + __half2float(bias[c0 + 2 * j + 1]), act);
    }
    o.h[j] = __floats2half2_rn(v0, v1);
  }
  *reinterpret_cast<uint4 *>(
      y + ((static_cast<long long>(n) * OH + oh) * OW + ow) * C + c0) = o.u;
}

// TMA-staged form: a block computes one output row x TW output columns x
// CB (<= 64) channels. One 4-D TMA box brings the KH input rows x
// ((TW-1)*SW + KW) columns x CB channels it needs into shared memory
// (zero-filled outside the image: the padding), the filter slice is staged
// tap-major beside it, and each thread computes PIX columns x 8 channels
// from shared memory with the same tap order and one mixed-precision FMA
// per multiply-add as depthwise_kernel (bit-identical results). (Packed
// fp32-pair FMAs on converted strips measured slower on B200.)
template <int KH, int KW, int SH, int SW, int PIX, int ACT>
__global__ void __launch_bounds__(256)
    depthwise_tma_kernel(const __grid_constant__ CUtensorMap xmap,
                         const half *__restrict__ w,
                         const half *__restrict__ bias, half *__restrict__ y,
                         int C, int H, int OH, int OW, int PH, int PW, int CB,
                         int TW, int tiles_w, int chunks, int act, int *err) {
  pdl_begin();
  constexpr int TAPS = KH * KW;
  constexpr int NCOL = (PIX - 1) * SW + KW;
  extern __shared__ __align__(128) uint8_t dwt_smem[];
  __shared__ uint64_t bar;
  __shared__ int failed;
  const int twin = (TW - 1) * SW + KW;
  half *xs = reinterpret_cast<half *>(dwt_smem);           // [KH][twin][CB]
  half *ws = xs + KH * twin * CB;                           // [TAPS][CB]
  // block -> (n, oh, column tile, channel chunk), last block first: the
  // producer wrote its highest rows last, and those are still in L2 (the
  // next kernel, walking upwards, then finds this one's lowest rows there).
  int b = gridDim.x - 1 - blockIdx.x;
  const int chunk = b % chunks;
  b /= chunks;
  const int tw = b % tiles_w;
  b /= tiles_w;
  const int oh = b % OH;
  const int n = b / OH;
  const int c0 = chunk * CB, ow0 = tw * TW;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    failed = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, static_cast<uint32_t>(KH * twin * CB * 2));
    tma_load_4d(xs, &xmap, &bar, c0, ow0 * SW - PW, oh * SH - PH, n);
  }
  for (int j = threadIdx.x; j < TAPS * CB; j += blockDim.x) {
    const int tap = j / CB, c = j - tap * CB; // w is [C][KH][KW]
    ws[j] = w[static_cast<long long>(c0 + c) * TAPS + tap];
  }
  volatile int no_abort = 0;
  const bool ok = mbar_wait(&bar, 0, &no_abort);
  if (!ok)
    failed = 1;
  __syncthreads();
  if (failed) {
    if (!ok)
      mbar_wait(&bar, 0, &no_abort);
    if (threadIdx.x == 0 && err)
      atomicCAS(err, 0, 7);
    return;
  }
  const int groups = CB >> 3;
  const int g = threadIdx.x % groups;
  const int t = threadIdx.x / groups;
  if (t * PIX >= TW)
    return;
  float acc[PIX][8];
#pragma unroll
  for (int p = 0; p < PIX; ++p)
#pragma unroll
    for (int j = 0; j < 8; ++j)
      acc[p][j] = 0.f;
  const int col0 = t * PIX * SW;
#pragma unroll
  for (int a = 0; a < KH; ++a) {
    // Rows outside the image (zero in shared memory) are skipped, as the
    // reference does.
    const int r = oh * SH - PH + a;
    if (r < 0 || r >= H)
      continue;
    const uint4 *row = reinterpret_cast<const uint4 *>(xs + (a * twin + col0) * CB) + g;
    uint4 strip[NCOL];
#pragma unroll
    for (int k = 0; k < NCOL; ++k)
      strip[k] = row[k * groups];
#pragma unroll
    for (int bq = 0; bq < KW; ++bq) {
      const uint4 wt = reinterpret_cast<const uint4 *>(ws + (a * KW + bq) * CB)[g];
#pragma unroll
      for (int p = 0; p < PIX; ++p) {
        const uint4 xv = strip[p * SW + bq];
        fma2_h(acc[p][0], acc[p][1], xv.x, wt.x);
        fma2_h(acc[p][2], acc[p][3], xv.y, wt.y);
        fma2_h(acc[p][4], acc[p][5], xv.z, wt.z);
        fma2_h(acc[p][6], acc[p][7], xv.w, wt.w);
      }
    }
  }
  float bv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    bv[j] = bias ? __half2float(bias[c0 + g * 8 + j]) : 0.f;
#pragma unroll
  for (int p = 0; p < PIX; ++p) {
    const int ow = ow0 + t * PIX + p;
    if (ow >= OW)
      break;
    Pack8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v0 = round_half(acc[p][2 * j]);
      float v1 = round_half(acc[p][2 * j + 1]);
      if (bias) {
        v0 = act_t<ACT>(v0 + bv[2 * j], act);
        v1 = act_t<ACT>(v1 + bv[2 * j + 1], act);
      }
      o.h[j] = __floats2half2_rn(v0, v1);
    }
    *reinterpret_cast<uint4 *>(
        y + ((static_cast<long long>(n) * OH + oh) * OW + ow) * C + c0 + g * 8) = o.u;
  }
}

template <int KH, int KW, int SH, int SW>
cudaError_t launch_dw_tma(const half *x, const half *w, const half *bias,
                          half *y, int batch, int C, int H, int W, int OH,
                          int OW, int PH, int PW, int act, cudaStream_t s,
                          bool *handled) {
  *handled = false;
  constexpr int PIX = 2;
  const int CB = C % 64 == 0 ? 64 : (C <= 64 ? C : 0);
  if (!CB || (reinterpret_cast<uintptr_t>(x) & 15))
    return cudaSuccess;
  const int groups = CB / 8;
  const int ntile = 256 / groups;     // column items per block
  const int TW = ntile * PIX;         // output columns per block
  const int twin = (TW - 1) * SW + KW;
  if (twin > 256)
    return cudaSuccess;
  const size_t smem =
      sizeof(half) * (static_cast<size_t>(KH) * twin * CB + KH * KW * CB);
  if (smem > 200 * 1024)
    return cudaSuccess;
  const int tiles_w = (OW + TW - 1) / TW;
  const int chunks = C / CB;
  const long long blocks = static_cast<long long>(batch) * OH * tiles_w * chunks;
  if (blocks >= (1LL << 31))
    return cudaSuccess;
  CUtensorMap map;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(C) * 2,
                           static_cast<cuuint64_t>(W) * C * 2,
                           static_cast<cuuint64_t>(H) * W * C * 2};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(CB), static_cast<cuuint32_t>(twin),
                       static_cast<cuuint32_t>(KH), 1};
  if (!encode_fp16_map(&map, x, 4, dims, strides, box, false))
    return cudaSuccess;
  auto kernel = act == kActRelu        ? depthwise_tma_kernel<KH, KW, SH, SW, PIX, kActRelu>
                : act == kActHardSwish ? depthwise_tma_kernel<KH, KW, SH, SW, PIX, kActHardSwish>
                                       : depthwise_tma_kernel<KH, KW, SH, SW, PIX, -1>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess)
    return e;
  *handled = true;
  launch_pdl(kernel, static_cast<unsigned>(blocks), 256, smem, s, map, w, bias, y, C, H, OH, OW, PH,
      PW, CB, TW, tiles_w, chunks, act, device_error_word());
  return cudaGetLastError();
}

// Multi-row tiled form: a block computes TH output rows x TW output columns
// x CB (<= 64) channels. One 4-D TMA box brings all the input it needs,
// ((TH-1)*SH + KH) rows x ((TW-1)*SW + KW) columns x CB channels (zero-filled
// outside the image: the padding), so each input row leaves HBM once per
// block instead of once per output row; the filter slice is staged tap-major
// beside it. A thread owns PIX consecutive output columns x 8 channels and
// walks the block's TH output rows; per input row it loads its strip of
// (PIX-1)*SW + KW 16-byte vectors once and reuses it for all KW taps. Sums
// follow the reference's tap order with one mixed-precision FMA per
// multiply-add (bit-identical to the other forms). The host sizes TW to
// divide the output width evenly (OW = 80 is one tile of 80 columns).
template <int KH, int KW, int SH, int SW, int PIX, int ACT>
__global__ void __launch_bounds__(256)
    depthwise_tile_kernel(const __grid_constant__ CUtensorMap xmap,
                          const half *__restrict__ w,
                          const half *__restrict__ bias, half *__restrict__ y,
                          int C, int H, int OH, int OW, int PH, int PW, int CB,
                          int TH, int TW, int tiles_h, int tiles_w, int chunks,
                          int act, int *err) {
  pdl_begin();
  constexpr int TAPS = KH * KW;
  constexpr int NCOL = (PIX - 1) * SW + KW;
  extern __shared__ __align__(128) uint8_t dwt_smem[];
  __shared__ uint64_t bar;
  __shared__ int failed;
  const int twin = (TW - 1) * SW + KW;
  const int rin = (TH - 1) * SH + KH;
  half *xs = reinterpret_cast<half *>(dwt_smem); // [rin][twin][CB]
  half *ws = xs + rin * twin * CB;                // [TAPS][CB]
  // block -> (n, row tile, column tile, channel chunk), last block first
  // (the producer's most recently written rows are the ones still in L2).
  int b = gridDim.x - 1 - blockIdx.x;
  const int chunk = b % chunks;
  b /= chunks;
  const int tw = b % tiles_w;
  b /= tiles_w;
  const int th = b % tiles_h;
  const int n = b / tiles_h;
  const int c0 = chunk * CB, ow0 = tw * TW, oh0 = th * TH;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    failed = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, static_cast<uint32_t>(rin * twin * CB * 2));
    tma_load_4d(xs, &xmap, &bar, c0, ow0 * SW - PW, oh0 * SH - PH, n);
  }
  // w is [C][KH][KW]: consecutive threads read consecutive filter values.
  for (int j = threadIdx.x; j < TAPS * CB; j += blockDim.x) {
    const int c = j / TAPS, tap = j - c * TAPS;
    ws[tap * CB + c] = w[static_cast<long long>(c0) * TAPS + j];
  }
  volatile int no_abort = 0;
  const bool ok = mbar_wait(&bar, 0, &no_abort);
  if (!ok)
    failed = 1;
  __syncthreads();
  if (failed) {
    if (!ok)
      mbar_wait(&bar, 0, &no_abort);
    if (threadIdx.x == 0 && err)
      atomicCAS(err, 0, 7);
    return;
  }
  const int groups = CB >> 3;
  const int g = threadIdx.x % groups;
  const int t = threadIdx.x / groups;
  if (t * PIX >= TW)
    return;
  const int col0 = t * PIX * SW;
  float bv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    bv[j] = bias ? __half2float(bias[c0 + g * 8 + j]) : 0.f;
  for (int rr = 0; rr < TH; ++rr) {
    const int oh = oh0 + rr;
    if (oh >= OH)
      break;
    float acc[PIX][8];
#pragma unroll
    for (int p = 0; p < PIX; ++p)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        acc[p][j] = 0.f;
#pragma unroll
    for (int a = 0; a < KH; ++a) {
      // Rows outside the image (zero in shared memory) are skipped, as the
      // reference does.
      const int r = oh * SH - PH + a;
      if (r < 0 || r >= H)
        continue;
      const uint4 *row =
          reinterpret_cast<const uint4 *>(xs + ((rr * SH + a) * twin + col0) * CB) + g;
      uint4 strip[NCOL];
#pragma unroll
      for (int k = 0; k < NCOL; ++k)
        strip[k] = row[k * groups];
#pragma unroll
      for (int bq = 0; bq < KW; ++bq) {
        const uint4 wt = reinterpret_cast<const uint4 *>(ws + (a * KW + bq) * CB)[g];
#pragma unroll
        for (int p = 0; p < PIX; ++p) {
          const uint4 xv = strip[p * SW + bq];
          fma2_h(acc[p][0], acc[p][1], xv.x, wt.x);
          fma2_h(acc[p][2], acc[p][3], xv.y, wt.y);
          fma2_h(acc[p][4], acc[p][5], xv.z, wt.z);
          fma2_h(acc[p][6], acc[p][7], xv.w, wt.w);
        }
      }
    }
    half *yrow = y + (static_cast<long long>(n) * OH + oh) * OW * C + c0 + g * 8;
#pragma unroll
    for (int p = 0; p < PIX; ++p) {
      const int ow = ow0 + t * PIX + p;
      if (ow >= OW)
        break;
      Pack8 o;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v0 = round_half(acc[p][2 * j]);
        float v1 = round_half(acc[p][2 * j + 1]);
        if (bias) {
          v0 = act_t<ACT>(v0 + bv[2 * j], act);
          v1 = act_t<ACT>(v1 + bv[2 * j + 1], act);
        }
        o.h[j] = __floats2half2_rn(v0, v1);
      }
      *reinterpret_cast<uint4 *>(yrow + static_cast<long long>(ow) * C) = o.u;
    }
  }
}

// Tile shape for depthwise_tile_kernel: the fewest column tiles of at most
// tw_max columns (TW a multiple of PIX, split evenly), then the most output
// rows whose input box fits smem_max bytes, split evenly over the row tiles.
struct DwTile {
  int CB = 0, TW = 0, TH = 0, tiles_w = 0, tiles_h = 0, threads = 0;
  size_t smem = 0;
};

inline DwTile pick_dw_tile(int C, int OH, int OW, int KH, int KW, int SH, int SW,
                           int PIX, int tw_req, int th_req) {
  DwTile t;
  t.CB = C % 64 == 0 ? 64 : (C <= 64 ? C : 0);
  if (!t.CB)
    return t;
  const int groups = t.CB / 8;
  const int tw_max = tw_req > 0 ? tw_req : std::min(256 / groups * PIX, 96);
  t.tiles_w = (OW + tw_max - 1) / tw_max;
  t.TW = ((OW + t.tiles_w - 1) / t.tiles_w + PIX - 1) / PIX * PIX;
  t.threads = groups * (t.TW / PIX);
  const int twin = (t.TW - 1) * SW + KW;
  if (t.threads > 256 || twin > 256) {
    t.CB = 0;
    return t;
  }
  const size_t row_bytes = static_cast<size_t>(twin) * t.CB * 2;
  const size_t wbytes = static_cast<size_t>(KH) * KW * t.CB * 2;
  const size_t smem_max = 76 * 1024;
  int th = th_req > 0 ? th_req : 1;
  if (th_req <= 0)
    while (th < OH && th < 16 &&
           static_cast<size_t>(th * SH + KH) * row_bytes + wbytes <= smem_max)
      ++th;
  t.tiles_h = (OH + th - 1) / th;
  t.TH = (OH + t.tiles_h - 1) / t.tiles_h;
  const int rin = (t.TH - 1) * SH + KH;
  if (rin > 256) {
    t.CB = 0;
    return t;
  }
  t.smem = rin * row_bytes + wbytes;
  return t;
}

template <int KH, int KW, int SH, int SW>
cudaError_t launch_dw_tile(const half *x, const half *w, const half *bias,
                           half *y, int batch, int C, int H, int W, int OH,
                           int OW, int PH, int PW, int act, cudaStream_t s,
                           bool *handled, int tw_req = 0, int th_req = 0) {
  *handled = false;
  constexpr int PIX = 4;
  if (reinterpret_cast<uintptr_t>(x) & 15)
    return cudaSuccess;
  const DwTile t = pick_dw_tile(C, OH, OW, KH, KW, SH, SW, PIX, tw_req, th_req);
  if (!t.CB || t.smem > 200 * 1024)
    return cudaSuccess;
  const int chunks = C / t.CB;
  const long long blocks =
      static_cast<long long>(batch) * t.tiles_h * t.tiles_w * chunks;
  if (blocks >= (1LL << 31))
    return cudaSuccess;
  const int twin = (t.TW - 1) * SW + KW;
  const int rin = (t.TH - 1) * SH + KH;
  CUtensorMap map;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(C) * 2,
                           static_cast<cuuint64_t>(W) * C * 2,
                           static_cast<cuuint64_t>(H) * W * C * 2};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(t.CB), static_cast<cuuint32_t>(twin),
                       static_cast<cuuint32_t>(rin), 1};
  if (!encode_fp16_map(&map, x, 4, dims, strides, box, false))
    return cudaSuccess;
  auto kernel = act == kActRelu        ? depthwise_tile_kernel<KH, KW, SH, SW, PIX, kActRelu>
                : act == kActHardSwish ? depthwise_tile_kernel<KH, KW, SH, SW, PIX, kActHardSwish>
                                       : depthwise_tile_kernel<KH, KW, SH, SW, PIX, -1>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(t.smem));
  if (e != cudaSuccess)
    return e;
  *handled = true;
  launch_pdl(kernel, static_cast<unsigned>(blocks), t.threads, t.smem, s, map, w, bias, y, C, H, OH,
      OW, PH, PW, t.CB, t.TH, t.TW, t.tiles_h, t.tiles_w, chunks, act, device_error_word());
  return cudaGetLastError();
}

template <int KH, int KW, int SH, int SW>
cudaError_t launch_dw(const half *x, const half *w, const half *bias, half *y,
                      int batch, int C, int H, int W, int OH, int OW, int PH,
                      int PW, int act, cudaStream_t s) {
  // Two output columns per item keeps the kernel at <= 64 registers (four
  // resident blocks per SM) so enough loads are in flight to cover latency.
  constexpr int PIX = 2;
  const int tiles = (OW + PIX - 1) / PIX;
  const long long total = static_cast<long long>(batch) * OH * tiles * (C / 8);
  const size_t smem = static_cast<size_t>(C) * KH * KW * sizeof(half);
  if (smem > 200 * 1024 || total >= (1LL << 31))
    return cudaErrorInvalidValue;
  long long blocks = (total + kBlock - 1) / kBlock;
  const long long cap = static_cast<long long>(sm_count()) * 16;
  if (blocks > cap)
    blocks = cap;
  auto kernel = act == kActRelu
                    ? depthwise_kernel<KH, KW, SH, SW, PIX, kActRelu>
                : act == kActHardSwish
                    ? depthwise_kernel<KH, KW, SH, SW, PIX, kActHardSwish>
                    : depthwise_kernel<KH, KW, SH, SW, PIX, -1>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        static_cast<int>(smem));
    if (e != cudaSuccess)
      return e;
  }
  launch_pdl(kernel, static_cast<unsigned>(blocks), kBlock, smem, s, x, w, bias, y, batch, C, H, W,
      OH, OW, PH, PW, act, static_cast<uint32_t>(total), FastDiv(C / 8), FastDiv(tiles),
      FastDiv(OH));
  return cudaGetLastError();
}

// ---------------------------------------------------------- direct conv
// Thread = one output pixel x 8 output channels. Filter in shared memory as
// fp32, summed in (kh, kw, ci) order.
__global__ void __launch_bounds__(kBlock)
    direct_conv_kernel(const half *__restrict__ x, const half *__restrict__ w,
                       const half *__restrict__ bias, half *__restrict__ y,
                       int batch, int Ci, int H, int W, int Co, int OH, int OW,
                       int KH, int KW, int SH, int SW, int PH, int PW,
                       int act) {
  pdl_begin();
  extern __shared__ float wsm[];
  const int wn = Co * KH * KW * Ci;
  for (int j = threadIdx.x; j < wn; j += blockDim.x)
    wsm[j] = __half2float(w[j]);
  __syncthreads();
  const int groups = Co >> 3;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(batch) * OH * OW * groups;
  if (i >= total)
    return;
  const int g = static_cast<int>(i % groups);
  long long t = i / groups;
  const int ow = static_cast<int>(t % OW);
  t /= OW;
  const int oh = static_cast<int>(t % OH);
  const int n = static_cast<int>(t / OH);
  const int co0 = g * 8;
  const int kstride = KH * KW * Ci;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int a = 0; a < KH; ++a) {
    const int r = oh * SH - PH + a;
    if (r < 0 || r >= H)
      continue;
    for (int b = 0; b < KW; ++b) {
      const int c = ow * SW - PW + b;
      if (c < 0 || c >= W)
        continue;
      const half *px = x + ((static_cast<long long>(n) * H + r) * W + c) * Ci;
      const int tap = (a * KW + b) * Ci;
      for (int ci = 0; ci < Ci; ++ci) {
        const float xv = __half2float(px[ci]);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          acc[j] = fmaf(xv, wsm[(co0 + j) * kstride + tap + ci], acc[j]);
      }
    }
  }
  Pack8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v0 = round_half(acc[2 * j]);
    float v1 = round_half(acc[2 * j + 1]);
    if (bias) {
      v0 += __half2float(bias[co0 + 2 * j]);
      v1 += __half2float(bias[co0 + 2 * j + 1]);
    }
    o.h[j] = __floats2half2_rn(apply_act(v0, act), apply_act(v1, act));
  }
  *reinterpret_cast<uint4 *>(
      y + ((static_cast<long long>(n) * OH + oh) * OW + ow) * Co + co0) = o.u;
}

// Stem form: thread = one output pixel x all CO output channels. The filter
// sits in shared memory tap-major ([kh][kw][ci][co], fp32) so each tap's
// CO weights are read as broadcast float4s; 16-byte output stores.
template <int CO, int ACT>
__global__ void __launch_bounds__(kBlock)
    stem_conv_kernel(const half *__restrict__ x, const half *__restrict__ w,
                     const half *__restrict__ bias, half *__restrict__ y,
                     int batch, int Ci, int H, int W, int OH, int OW, int KH,
                     int KW, int SH, int SW, int PH, int PW, int act,
                     uint32_t total, FastDiv by_ow, FastDiv by_oh) {
  pdl_begin();
  extern __shared__ float wsm[];
  const int taps = KH * KW * Ci;
  for (int j = threadIdx.x; j < taps * CO; j += blockDim.x) {
    const int co = j / taps, k = j - co * taps; // w is [co][kh][kw][ci]
    wsm[k * CO + co] = __half2float(w[j]);
  }
  __syncthreads();
  const uint32_t p = blockIdx.x * blockDim.x + threadIdx.x; // below 2^31
  if (p >= total)
    return;
  const uint32_t r0 = by_ow.div(p);
  const int ow = static_cast<int>(p - r0 * by_ow.d);
  const uint32_t n0 = by_oh.div(r0);
  const int oh = static_cast<int>(r0 - n0 * by_oh.d);
  const long long n = n0;
  float acc[CO];
#pragma unroll
  for (int c = 0; c < CO; ++c)
    acc[c] = 0.f;
  for (int a = 0; a < KH; ++a) {
    const int r = oh * SH - PH + a;
    if (r < 0 || r >= H)
      continue;
    for (int b = 0; b < KW; ++b) {
      const int c = ow * SW - PW + b;
      if (c < 0 || c >= W)
        continue;
      const half *px = x + ((n * H + r) * W + c) * Ci;
      const float4 *wt = reinterpret_cast<const float4 *>(wsm + (a * KW + b) * Ci * CO);
      for (int ci = 0; ci < Ci; ++ci) {
        const float xv = __half2float(px[ci]);
#pragma unroll
        for (int q = 0; q < CO / 4; ++q) {
          const float4 wv = wt[ci * (CO / 4) + q];
          acc[4 * q] = fmaf(xv, wv.x, acc[4 * q]);
          acc[4 * q + 1] = fmaf(xv, wv.y, acc[4 * q + 1]);
          acc[4 * q + 2] = fmaf(xv, wv.z, acc[4 * q + 2]);
          acc[4 * q + 3] = fmaf(xv, wv.w, acc[4 * q + 3]);
        }
      }
    }
  }
  half *dst = y + static_cast<long long>(p) * CO;
#pragma unroll
  for (int g = 0; g < CO / 8; ++g) {
    Pack8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c0 = g * 8 + 2 * j;
      float v0 = round_half(acc[c0]), v1 = round_half(acc[c0 + 1]);
      if (bias) {
        v0 += __half2float(bias[c0]);
        v1 += __half2float(bias[c0 + 1]);
      }
      o.h[j] = __floats2half2_rn(act_t<ACT>(v0, act), act_t<ACT>(v1, act));
    }
    *reinterpret_cast<uint4 *>(dst + g * 8) = o.u;
  }
}

// Two horizontally adjacent output pixels per thread for small Ci (the
// stem): each filter tap's CO fp32 weights are read from shared memory once
// (broadcast) for both pixels, and the multiply-adds run as packed fp32
// pairs over output channels. Sum order per output is (kh, kw, ci) as in
// stem_conv_kernel, so results are bit-identical to it.
template <int CO, int ACT>
__global__ void __launch_bounds__(kBlock)
    stem_conv2_kernel(const half *__restrict__ x, const half *__restrict__ w,
                      const half *__restrict__ bias, half *__restrict__ y,
                      int Ci, int H, int W, int OH, int OW, int KH, int KW,
                      int SH, int SW, int PH, int PW, int act, uint32_t items,
                      FastDiv by_pairs, FastDiv by_oh) {
  pdl_begin();
  extern __shared__ float wsm[];
  const int taps = KH * KW * Ci;
  for (int j = threadIdx.x; j < taps * CO; j += blockDim.x) {
    const int co = j / taps, k = j - co * taps; // w is [co][kh][kw][ci]
    wsm[k * CO + co] = __half2float(w[j]);
  }
  __syncthreads();
  const uint32_t it = blockIdx.x * blockDim.x + threadIdx.x;
  if (it >= items)
    return;
  const uint32_t r0 = by_pairs.div(it);
  const int ow = static_cast<int>(it - r0 * by_pairs.d) * 2;
  const uint32_t n0 = by_oh.div(r0);
  const int oh = static_cast<int>(r0 - n0 * by_oh.d);
  const long long n = n0;
  const bool two = ow + 1 < OW;
  float2 acc0[CO / 2], acc1[CO / 2];
#pragma unroll
  for (int c = 0; c < CO / 2; ++c)
    acc0[c] = acc1[c] = make_float2(0.f, 0.f);
  for (int a = 0; a < KH; ++a) {
    const int r = oh * SH - PH + a;
    if (r < 0 || r >= H)
      continue;
    for (int b = 0; b < KW; ++b) {
      const int c0 = ow * SW - PW + b, c1 = c0 + SW;
      const bool in0 = c0 >= 0 && c0 < W, in1 = two && c1 >= 0 && c1 < W;
      if (!in0 && !in1)
        continue;
      const half *p0 = x + ((n * H + r) * W + c0) * Ci;
      const half *p1 = p0 + static_cast<long long>(SW) * Ci;
      const float4 *wt = reinterpret_cast<const float4 *>(wsm + (a * KW + b) * Ci * CO);
      for (int ci = 0; ci < Ci; ++ci) {
        const float x0 = in0 ? __half2float(p0[ci]) : 0.f;
        const float x1 = in1 ? __half2float(p1[ci]) : 0.f;
        const float2 xx0 = make_float2(x0, x0), xx1 = make_float2(x1, x1);
#pragma unroll
        for (int q = 0; q < CO / 4; ++q) {
          const float4 wv = wt[ci * (CO / 4) + q];
          const float2 wlo = make_float2(wv.x, wv.y), whi = make_float2(wv.z, wv.w);
          if (in0) {
            ffma2(acc0[2 * q], xx0, wlo);
            ffma2(acc0[2 * q + 1], xx0, whi);
          }
          if (in1) {
            ffma2(acc1[2 * q], xx1, wlo);
            ffma2(acc1[2 * q + 1], xx1, whi);
          }
        }
      }
    }
  }
  auto store = [&](const float2 (&acc)[CO / 2], int col) {
    half *dst = y + ((n * OH + oh) * OW + col) * CO;
#pragma unroll
    for (int g = 0; g < CO / 8; ++g) {
      Pack8 o;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c0 = g * 8 + 2 * j;
        float v0 = round_half(acc[c0 / 2].x), v1 = round_half(acc[c0 / 2].y);
        if (bias) {
          v0 += __half2float(bias[c0]);
          v1 += __half2float(bias[c0 + 1]);
        }
        o.h[j] = __floats2half2_rn(act_t<ACT>(v0, act), act_t<ACT>(v1, act));
      }
      *reinterpret_cast<uint4 *>(dst + g * 8) = o.u;
    }
  };
  store(acc0, ow);
  if (two)
    store(acc1, ow + 1);
}

// ----------------------------------------------------------------- pool
__global__ void __launch_bounds__(kBlock)
    pool_nhwc_vec_kernel(const half *__restrict__ x, half *__restrict__ y,
                         int batch, int C, int H, int W, int OH, int OW,
                         int KH, int KW, int SH, int SW, int PH, int PW,
                         bool maximum) {
  pdl_begin();
  const int groups = C >> 3;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(batch) * OH * OW * groups;
  if (i >= total)
    return;
  const int g = static_cast<int>(i % groups);
  long long t = i / groups;
  const int ow = static_cast<int>(t % OW);
  t /= OW;
  const int oh = static_cast<int>(t % OH);
  const int n = static_cast<int>(t / OH);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    acc[j] = maximum ? -INFINITY : 0.f;
  int valid = 0;
  const int r0 = oh * SH - PH, q0 = ow * SW - PW;
  for (int a = 0; a < KH; ++a) {
    for (int b = 0; b < KW; ++b) {
      const int r = r0 + a, c = q0 + b;
      if (r < 0 || r >= H || c < 0 || c >= W)
        continue;
      Pack8 v;
      v.u = __ldg(reinterpret_cast<const uint4 *>(
          x + ((static_cast<long long>(n) * H + r) * W + c) * C + g * 8));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(v.h[j]);
        acc[2 * j] = maximum ? fmaxf(acc[2 * j], f.x) : acc[2 * j] + f.x;
        acc[2 * j + 1] =
            maximum ? fmaxf(acc[2 * j + 1], f.y) : acc[2 * j + 1] + f.y;
      }
      ++valid;
    }
  }
  Pack8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    o.h[j] = __floats2half2_rn(maximum ? acc[2 * j] : acc[2 * j] / valid,
                               maximum ? acc[2 * j + 1]
                                       : acc[2 * j + 1] / valid);
  *reinterpret_cast<uint4 *>(y + i * 8) = o.u;
}

// Unpadded fixed-window form (the recognizer's 3x2/3x2 average and the
// stem's 2x2/1 max): every tap is in bounds, so all loads issue together.
template <int KH, int KW, int SH, int SW, bool MAXIMUM>
__global__ void __launch_bounds__(kBlock)
    pool_fixed_kernel(const half *__restrict__ x, half *__restrict__ y,
                      int batch, int C, int H, int W, int OH, int OW,
                      FastDiv by_groups, FastDiv by_ow, FastDiv by_oh) {
  pdl_begin();
  const int groups = C >> 3;
  // Last block first: the producer's most recently written rows are the ones
  // still in L2.
  long long i = static_cast<long long>(gridDim.x - 1 - blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(batch) * OH * OW * groups;
  if (i >= total)
    return;
  int g, ow, oh;
  long long n;
  if (total < (1LL << 31)) {
    // 32-bit multiply-shift division (a 64-bit divide costs dozens of
    // instructions per 16-byte output).
    const uint32_t i32 = static_cast<uint32_t>(i);
    const uint32_t p = by_groups.div(i32);
    g = static_cast<int>(i32 - p * by_groups.d);
    const uint32_t r = by_ow.div(p);
    ow = static_cast<int>(p - r * by_ow.d);
    const uint32_t q = by_oh.div(r);
    oh = static_cast<int>(r - q * by_oh.d);
    n = q;
  } else {
    g = static_cast<int>(i % groups);
    long long t = i / groups;
    ow = static_cast<int>(t % OW);
    t /= OW;
    oh = static_cast<int>(t % OH);
    n = t / OH;
  }
  const half *base = x + ((n * H + oh * SH) * W + ow * SW) * C + g * 8;
  Pack8 v[KH * KW];
#pragma unroll
  for (int a = 0; a < KH; ++a)
#pragma unroll
    for (int b = 0; b < KW; ++b)
      v[a * KW + b].u = __ldg(reinterpret_cast<const uint4 *>(
          base + (static_cast<long long>(a) * W + b) * C));
  Pack8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 acc = __half22float2(v[0].h[j]);
#pragma unroll
    for (int k = 1; k < KH * KW; ++k) {
      const float2 f = __half22float2(v[k].h[j]);
      acc.x = MAXIMUM ? fmaxf(acc.x, f.x) : acc.x + f.x;
      acc.y = MAXIMUM ? fmaxf(acc.y, f.y) : acc.y + f.y;
    }
    if (!MAXIMUM) {
      acc.x /= KH * KW;
      acc.y /= KH * KW;
    }
    o.h[j] = __floats2half2_rn(acc.x, acc.y);
  }
  *reinterpret_cast<uint4 *>(y + i * 8) = o.u;
}

__global__ void __launch_bounds__(kBlock)
    pool_scalar_kernel(const half *__restrict__ x, half *__restrict__ y,
                       long long total, int C, int H, int W, int OH, int OW,
                       int KH, int KW, int SH, int SW, int PH, int PW,
                       bool maximum, bool nhwc) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  int c, ow, oh;
  long long plane;
  if (nhwc) {
    c = static_cast<int>(i % C);
    long long p = i / C;
    ow = static_cast<int>(p % OW);
    oh = static_cast<int>((p / OW) % OH);
    plane = p / (static_cast<long long>(OW) * OH); // batch index
  } else {
    ow = static_cast<int>(i % OW);
    oh = static_cast<int>((i / OW) % OH);
    plane = i / (static_cast<long long>(OW) * OH);
    c = 0;
  }
  float v = maximum ? -INFINITY : 0.f;
  int valid = 0;
  for (int a = 0; a < KH; ++a)
    for (int b = 0; b < KW; ++b) {
      const int r = oh * SH - PH + a, q = ow * SW - PW + b;
      if (r < 0 || r >= H || q < 0 || q >= W)
        continue;
      const long long idx =
          nhwc ? ((plane * H + r) * W + q) * C + c : (plane * H + r) * W + q;
      const float z = __half2float(x[idx]);
      v = maximum ? fmaxf(v, z) : v + z;
      ++valid;
    }
  y[i] = __float2half_rn(maximum ? v : v / valid);
}

// ------------------------------------------------------------------ pad
__global__ void __launch_bounds__(kBlock)
    pad_kernel(const half *__restrict__ x, half *__restrict__ y,
               long long total, int C, int H, int W, int OH, int OW, int PH,
               int PW, bool vec) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  // vec: NHWC, one 8-channel group per thread. !vec with C==1: NCHW planes.
  const int groups = vec ? C / 8 : C;
  const int g = static_cast<int>(i % groups);
  long long p = i / groups;
  const int ow = static_cast<int>(p % OW);
  const int oh = static_cast<int>((p / OW) % OH);
  const long long n = p / (static_cast<long long>(OW) * OH);
  const int r = oh - PH, c = ow - PW;
  const bool in = r >= 0 && r < H && c >= 0 && c < W;
  const long long src = ((n * H + r) * W + c) * C;
  if (vec) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (in)
      v = __ldg(reinterpret_cast<const uint4 *>(x + src + g * 8));
    *reinterpret_cast<uint4 *>(y + i * 8) = v;
  } else {
    y[i] = in ? x[src + g] : __float2half_rn(0.f);
  }
}

// --------------------------------------------------------------- resize
__global__ void __launch_bounds__(kBlock)
    resize_nhwc_kernel(const half *__restrict__ x,
                       const half *__restrict__ addend, half *__restrict__ y,
                       long long total, int C, int H, int W, int OH, int OW,
                       float sh, float sw, bool vec) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const int groups = vec ? C / 8 : C;
  const int g = static_cast<int>(i % groups);
  long long p = i / groups;
  const int ow = static_cast<int>(p % OW);
  const int oh = static_cast<int>((p / OW) % OH);
  const long long n = p / (static_cast<long long>(OW) * OH);
  const int r = min(static_cast<int>(floorf(oh / sh)), H - 1);
  const int c = min(static_cast<int>(floorf(ow / sw)), W - 1);
  const long long src = ((n * H + r) * W + c) * C;
  if (vec) {
    Pack8 v;
    v.u = __ldg(reinterpret_cast<const uint4 *>(x + src + g * 8));
    if (addend) {
      Pack8 a;
      a.u = __ldg(reinterpret_cast<const uint4 *>(addend + i * 8));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(v.h[j]), e = __half22float2(a.h[j]);
        v.h[j] = __floats2half2_rn(f.x + e.x, f.y + e.y);
      }
    }
    *reinterpret_cast<uint4 *>(y + i * 8) = v.u;
  } else {
    float v = __half2float(x[src + g]);
    if (addend)
      v += __half2float(addend[i]);
    y[i] = __float2half_rn(v);
  }
}

// FPN tail in one pass: y[n, h, w, :] = [src_0(n, h, w) | src_1 up | ...],
// each source nearest-upsampled by its own scale with the resize kernel's
// mapping (src = min(floor(dst / scale), n - 1)), so the result equals the
// chain of resize_nearest_nhwc + concat launches bit for bit while the
// concatenated tensor is written once and no intermediate is. Thread = one
// 16-byte group of 8 output channels; consecutive threads walk a pixel's
// channel groups.
__global__ void __launch_bounds__(kBlock)
    upsample_concat_kernel(const __grid_constant__ UpcatArgs a, half *__restrict__ y,
                           uint32_t total, FastDiv by_groups, FastDiv by_ow, FastDiv by_oh) {
  pdl_begin();
  // The source table goes to shared memory once per block: lanes of a warp
  // pick different sources, and lane-dependent indices into the parameter
  // block (or selecting through all of it per thread) stall on its loads.
  __shared__ const half *s_src[kUpcatMax];
  __shared__ int s_dim[3][kUpcatMax];
  __shared__ float s_scale[2][kUpcatMax];
  if (threadIdx.x < kUpcatMax && static_cast<int>(threadIdx.x) < a.n) {
    const int k = threadIdx.x;
    s_src[k] = a.src[k];
    s_dim[0][k] = a.C[k];
    s_dim[1][k] = a.H[k];
    s_dim[2][k] = a.W[k];
    s_scale[0][k] = a.sh[k];
    s_scale[1][k] = a.sw[k];
  }
  __syncthreads();
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const uint32_t p = by_groups.div(i);
  int c = static_cast<int>(i - p * by_groups.d) * 8;
  const uint32_t r = by_ow.div(p);
  const int ow = static_cast<int>(p - r * by_ow.d);
  const uint32_t n = by_oh.div(r);
  const int oh = static_cast<int>(r - n * by_oh.d);
  int k = 0;
  while (k + 1 < a.n && c >= s_dim[0][k]) {
    c -= s_dim[0][k];
    ++k;
  }
  const int C = s_dim[0][k], H = s_dim[1][k], W = s_dim[2][k];
  const int sr = min(static_cast<int>(floorf(oh / s_scale[0][k])), H - 1);
  const int sc = min(static_cast<int>(floorf(ow / s_scale[1][k])), W - 1);
  const half *src = s_src[k] + ((static_cast<long long>(n) * H + sr) * W + sc) * C + c;
  reinterpret_cast<uint4 *>(y)[i] = __ldg(reinterpret_cast<const uint4 *>(src));
}

// 32-bit-index form of resize_nhwc_kernel for 16-byte channel groups
// (total < 2^31): the pixel/row/image split by multiply-shift division
// instead of 64-bit divides; same source mapping and arithmetic.
__global__ void __launch_bounds__(kBlock)
    resize_nhwc_vec_kernel(const half *__restrict__ x, const half *__restrict__ addend,
                           half *__restrict__ y, uint32_t total, int C, int H, int W,
                           FastDiv by_groups, FastDiv by_ow, FastDiv by_oh, float sh, float sw) {
  pdl_begin();
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const uint32_t p = by_groups.div(i);
  const int g = static_cast<int>(i - p * by_groups.d);
  const uint32_t rr = by_ow.div(p);
  const int ow = static_cast<int>(p - rr * by_ow.d);
  const uint32_t n = by_oh.div(rr);
  const int oh = static_cast<int>(rr - n * by_oh.d);
  const int r = min(static_cast<int>(floorf(oh / sh)), H - 1);
  const int c = min(static_cast<int>(floorf(ow / sw)), W - 1);
  const long long src = ((static_cast<long long>(n) * H + r) * W + c) * C;
  Pack8 v;
  v.u = __ldg(reinterpret_cast<const uint4 *>(x + src + g * 8));
  if (addend) {
    Pack8 a;
    a.u = __ldg(reinterpret_cast<const uint4 *>(addend) + i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(v.h[j]), e = __half22float2(a.h[j]);
      v.h[j] = __floats2half2_rn(f.x + e.x, f.y + e.y);
    }
  }
  reinterpret_cast<uint4 *>(y)[i] = v.u;
}

__global__ void __launch_bounds__(kBlock)
    resize_nchw_kernel(const half *__restrict__ x, half *__restrict__ y,
                       long long total, int H, int W, int OH, int OW, float sh,
                       float sw) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const int ow = static_cast<int>(i % OW);
  const int oh = static_cast<int>((i / OW) % OH);
  const long long plane = i / (static_cast<long long>(OW) * OH);
  const int r = min(static_cast<int>(floorf(oh / sh)), H - 1);
  const int c = min(static_cast<int>(floorf(ow / sw)), W - 1);
  y[i] = x[(plane * H + r) * W + c];
}

// --------------------------------------------------------------- concat
__global__ void __launch_bounds__(kBlock)
    concat_kernel(const half *__restrict__ a, const half *__restrict__ b,
                  half *__restrict__ y, long long total, int na, int nb,
                  bool vec) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const int width = na + nb;
  const long long row = i / width;
  const int col = static_cast<int>(i % width);
  if (vec) {
    const uint4 *src = col < na ? reinterpret_cast<const uint4 *>(a) + row * na + col
                                : reinterpret_cast<const uint4 *>(b) + row * nb + (col - na);
    reinterpret_cast<uint4 *>(y)[i] = __ldg(src);
  } else {
    y[i] = col < na ? a[row * na + col] : b[row * nb + col - na];
  }
}

// ------------------------------------------------------------ transpose
__global__ void transpose_kernel(const half *__restrict__ x,
                                 half *__restrict__ y, int rows, int cols) {
  pdl_begin();
  __shared__ half tile[32][34];
  const long long base = static_cast<long long>(blockIdx.z) * rows * cols;
  int c = blockIdx.x * 32 + threadIdx.x;
  int r = blockIdx.y * 32 + threadIdx.y;
  for (int j = 0; j < 32; j += 8)
    if (c < cols && r + j < rows)
      tile[threadIdx.y + j][threadIdx.x] =
          x[base + static_cast<long long>(r + j) * cols + c];
  __syncthreads();
  c = blockIdx.y * 32 + threadIdx.x;
  r = blockIdx.x * 32 + threadIdx.y;
  for (int j = 0; j < 32; j += 8)
    if (c < rows && r + j < cols)
      y[base + static_cast<long long>(r + j) * rows + c] =
          tile[threadIdx.x][threadIdx.y + j];
}

__device__ __forceinline__ long long locate(long long i, const Gather &g) {
  long long off = g.offset;
  for (int d = g.rank - 1; d >= 0; --d) {
    off += (i % g.shape[d]) * g.stride[d];
    i /= g.shape[d];
  }
  return off;
}

__global__ void __launch_bounds__(kBlock)
    gather_kernel(const half *__restrict__ x, half *__restrict__ y,
                  long long n, Gather g) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n)
    y[i] = x[locate(i, g)];
}

__device__ __forceinline__ float binop(float x, float z, int op) {
  return op == 0   ? x + z
         : op == 1 ? x - z
         : op == 2 ? x * z
         : op == 3 ? x / z
                   : powf(x, z);
}

__global__ void __launch_bounds__(kBlock)
    binary_kernel(const half *__restrict__ a, const half *__restrict__ b,
                  half *__restrict__ y, long long n, Gather ga, Gather gb,
                  int op) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n)
    y[i] = __float2half_rn(binop(__half2float(a[locate(i, ga)]),
                                 __half2float(b[locate(i, gb)]), op));
}

__device__ __forceinline__ long long flat(long long i, int d, int m) {
  if (m == 1)
    return 0;
  if (d != 1)
    i /= d;
  if (m > 1)
    i %= m;
  return i;
}

__global__ void __launch_bounds__(kBlock)
    binary_flat_kernel(const half *__restrict__ a, const half *__restrict__ b,
                       half *__restrict__ y, long long n, int ad, int am,
                       int bd, int bm, int op) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n)
    y[i] = __float2half_rn(binop(__half2float(a[flat(i, ad, am)]),
                                 __half2float(b[flat(i, bd, bm)]), op));
}

__global__ void __launch_bounds__(kBlock)
    unary_kernel(const half *__restrict__ x, half *__restrict__ y, long long n,
                 int op, float alpha, float beta) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n)
    return;
  const float v = __half2float(x[i]);
  float r;
  switch (op) {
  case 0:
    r = fmaxf(v, 0.f);
    break;
  case 1:
    r = 1.f / (1.f + expf(-v));
    break;
  case 2:
    r = fminf(1.f, fmaxf(0.f, alpha * v + beta));
    break;
  case 3:
    r = erff(v);
    break;
  case 4:
    r = sqrtf(v);
    break;
  default:
    r = v;
  }
  y[i] = __float2half_rn(r);
}

__global__ void __launch_bounds__(kBlock)
    copy_input_f32_kernel(const float *__restrict__ x, half *__restrict__ y,
                          size_t valid, size_t total) {
  pdl_begin();
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < total)
    y[i] = i < valid ? __float2half_rn(x[i]) : __float2half_rn(0.f);
}

// NHWC (valid images) -> NCHW, zero for images >= valid.
__global__ void __launch_bounds__(kBlock)
    copy_input_nhwc_kernel(const half *__restrict__ x, half *__restrict__ y,
                           int valid, long long total, int C, int H, int W) {
  pdl_begin();
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const int w = static_cast<int>(i % W);
  const int h = static_cast<int>((i / W) % H);
  const int c = static_cast<int>((i / (static_cast<long long>(W) * H)) % C);
  const long long n = i / (static_cast<long long>(W) * H * C);
  y[i] = n < valid ? x[((n * H + h) * W + w) * C + c] : __float2half_rn(0.f);
}

__global__ void __launch_bounds__(kBlock)
    half_to_float_kernel(const half *__restrict__ x, float *__restrict__ y,
                         size_t n) {
  pdl_begin();
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n)
    y[i] = __half2float(x[i]);
}

// Thread = one pixel: reads its C values from the C planes (coalesced per
// plane across the warp), writes C consecutive halves.
__global__ void __launch_bounds__(kBlock)
    nchw_to_nhwc_kernel(const float *__restrict__ x, half *__restrict__ y,
                        int valid, long long pixels, int C, int HW) {
  pdl_begin();
  long long p = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= pixels)
    return;
  const long long n = p / HW;
  const int s = static_cast<int>(p - n * HW);
  half *dst = y + p * C;
  if (n >= valid) {
    for (int c = 0; c < C; ++c)
      dst[c] = __float2half_rn(0.f);
    return;
  }
  const float *src = x + n * C * HW + s;
  for (int c = 0; c < C; ++c)
    dst[c] = __float2half_rn(__ldg(src + static_cast<long long>(c) * HW));
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

} // namespace

cudaError_t nchw_f32_to_nhwc_f16(const float *x, half *y, int valid, int batch,
                                 int C, int H, int W, cudaStream_t s) {
  const long long pixels = static_cast<long long>(batch) * H * W;
  if (pixels <= 0)
    return cudaSuccess;
  launch_pdl(nchw_to_nhwc_kernel, blocks_for(pixels), kBlock, 0, s, x, y, valid, pixels, C, H * W);
  return cudaGetLastError();
}

cudaError_t depthwise(const half *x, const half *w, const half *bias, half *y,
                      int batch, int C, int H, int W, int OH, int OW, int KH,
                      int KW, int SH, int SW, int PH, int PW, int act,
                      cudaStream_t s) {
  if (batch <= 0 || OH <= 0 || OW <= 0)
    return cudaSuccess;
  if (C % 8 || !al16(x) || !al16(y))
    return cudaErrorInvalidValue;
#define PB2_DW(kh, kw, sh, sw)                                                 \
  if (KH == kh && KW == kw && SH == sh && SW == sw) {                          \
    bool handled = false;                                                      \
    cudaError_t e = launch_dw_tile<kh, kw, sh, sw>(x, w, bias, y, batch, C, H, \
                                                   W, OH, OW, PH, PW, act, s,  \
                                                   &handled);                  \
    if (handled || e != cudaSuccess)                                           \
      return e;                                                                \
    e = launch_dw_tma<kh, kw, sh, sw>(x, w, bias, y, batch, C, H, W, OH, OW,   \
                                      PH, PW, act, s, &handled);               \
    if (handled || e != cudaSuccess)                                           \
      return e;                                                                \
    return launch_dw<kh, kw, sh, sw>(x, w, bias, y, batch, C, H, W, OH, OW,    \
                                     PH, PW, act, s);                          \
  }
  PB2_DW(3, 3, 1, 1)
  PB2_DW(3, 3, 2, 2)
  PB2_DW(3, 3, 2, 1)
  PB2_DW(5, 5, 1, 1)
  PB2_DW(5, 5, 2, 2)
  PB2_DW(1, 7, 1, 1)
  PB2_DW(9, 9, 1, 1)
#undef PB2_DW
  const long long total = static_cast<long long>(batch) * OH * OW * (C / 8);
  launch_pdl(depthwise_generic_kernel, blocks_for(total), kBlock, 0, s, x, w, bias, y, batch, C, H,
      W, OH, OW, KH, KW, SH, SW, PH, PW, act);
  return cudaGetLastError();
}

// Stem on the tensor cores: a 3x3 stride-2 pad-1 convolution of a Ci <= 4
// image equals a 2x2 stride-1 convolution (pad 1 at the top/left) of its
// space-to-depth rearrangement: block pixel (R, C) holds the 2x2 input
// pixels (2R + dr, 2C + dc) as channel (dr*2 + dc)*4 + c (16 channels, 32
// bytes, zero past Ci and past the image edge). Filter tap (kh, kw) of the
// 3x3 conv becomes tap (a, b) = ((kh + 1) / 2, (kw + 1) / 2) of the 2x2 conv
// at sub-pixel (dr, dc) = ((kh + 1) % 2, (kw + 1) % 2).
namespace {
__global__ void __launch_bounds__(kBlock)
    space_to_depth2_kernel(const half *__restrict__ x, uint4 *__restrict__ y,
                           int Ci, int H, int W, int H2, int W2, uint32_t total,
                           FastDiv by_w2, FastDiv by_h2) {
  pdl_begin();
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total)
    return;
  const uint32_t r = by_w2.div(i);
  const int bc = static_cast<int>(i - r * by_w2.d);
  const uint32_t n = by_h2.div(r);
  const int br = static_cast<int>(r - n * by_h2.d);
  half v[16];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int row = 2 * br + (q >> 1), col = 2 * bc + (q & 1);
    const bool in = row < H && col < W;
    const half *px = x + ((static_cast<long long>(n) * H + row) * W + col) * Ci;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      v[q * 4 + c] = in && c < Ci ? px[c] : __float2half_rn(0.f);
  }
  const uint4 *vv = reinterpret_cast<const uint4 *>(v);
  y[2ull * i] = vv[0];
  y[2ull * i + 1] = vv[1];
}

__global__ void __launch_bounds__(kBlock)
    stem_s2d_pack_kernel(const half *__restrict__ w, half *__restrict__ wp,
                         int Co, int Ci) {
  pdl_begin();
  // wp [Co][2][2][16] from w [Co][3][3][Ci] (OHWI)
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= Co * 64)
    return;
  const int co = i / 64, rem = i % 64;
  const int tap = rem / 16, ch = rem % 16;
  const int a = tap >> 1, b = tap & 1, q = ch >> 2, c = ch & 3;
  const int dr = q >> 1, dc = q & 1;
  const int kh = 2 * a + dr - 1, kw = 2 * b + dc - 1;
  const bool ok = kh >= 0 && kh < 3 && kw >= 0 && kw < 3 && c < Ci;
  wp[i] = ok ? w[((static_cast<long long>(co) * 3 + kh) * 3 + kw) * Ci + c]
             : __float2half_rn(0.f);
}

} // namespace

cudaError_t stem_s2d_pack(const half *w, half *wp, int Co, int Ci,
                          cudaStream_t s) {
  if (Co <= 0 || Ci <= 0 || Ci > 4)
    return cudaErrorInvalidValue;
  launch_pdl(stem_s2d_pack_kernel, blocks_for(static_cast<long long>(Co) * 64), kBlock, 0, s, w, wp,
      Co, Ci);
  return cudaGetLastError();
}

size_t stem_s2d_scratch_bytes(int batch, int H, int W) {
  return static_cast<size_t>(batch) * ((H + 1) / 2) * ((W + 1) / 2) * 32;
}

cudaError_t stem_conv_s2d(const half *x, const half *wp, const half *bias,
                          half *y, half *scratch, int batch, int Ci, int H,
                          int W, int Co, int act, cudaStream_t s) {
  if (batch <= 0 || H <= 0 || W <= 0)
    return cudaSuccess;
  if (Ci <= 0 || Ci > 4 || Co % 8 || !al16(scratch) || !al16(wp))
    return cudaErrorInvalidValue;
  const int H2 = (H + 1) / 2, W2 = (W + 1) / 2;
  const long long total = static_cast<long long>(batch) * H2 * W2;
  if (total >= (1LL << 31))
    return cudaErrorInvalidValue;
  launch_pdl(space_to_depth2_kernel, blocks_for(total), kBlock, 0, s, x,
      reinterpret_cast<uint4 *>(scratch), Ci, H, W, H2, W2, static_cast<uint32_t>(total),
      FastDiv(W2), FastDiv(H2));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return e;
  GemmEpilogue epi;
  epi.bias = bias;
  epi.out = y;
  epi.ldo = Co;
  epi.act = act;
  ConvShape cs{batch, H2, W2, 16, Co, 2, 2, 1, 1};
  cs.out_h = H2;
  cs.out_w = W2;
  return tc_conv(scratch, wp, cs, epi, s);
}

cudaError_t direct_conv(const half *x, const half *w, const half *bias,
                        half *y, int batch, int Ci, int H, int W, int Co,
                        int OH, int OW, int KH, int KW, int SH, int SW, int PH,
                        int PW, int act, cudaStream_t s) {
  if (batch <= 0 || OH <= 0 || OW <= 0)
    return cudaSuccess;
  const size_t smem = sizeof(float) * static_cast<size_t>(Co) * KH * KW * Ci;
  if (Co % 8 || !al16(y) || smem > 48 * 1024)
    return cudaErrorInvalidValue;
  const long long pixels = static_cast<long long>(batch) * OH * OW;
  const long long pairs = static_cast<long long>(batch) * OH * ((OW + 1) / 2);
  // The HGNet stem (3x3 / s2 / p1 over 3 channels) runs on the tensor cores.
  if (Ci == 3 && KH == 3 && KW == 3 && SH == 2 && SW == 2 && PH == 1 && PW == 1 && OH == (H + 1) / 2 &&
      OW == (W + 1) / 2) {
    const cudaError_t e = stem_conv_tc(x, w, bias, y, batch, H, W, Co, act, s);
    if (e != cudaErrorNotSupported)
      return e;
  }
  if (Ci <= 4 && (Co == 16 || Co == 32 || Co == 48) && pairs < (1LL << 31)) {
    const int per_row = (OW + 1) / 2;
#define PB2_STEM2(co)                                                          \
  if (Co == co) {                                                              \
    launch_pdl(act == kActRelu ? stem_conv2_kernel<co, kActRelu>               \
                               : stem_conv2_kernel<co, -1>,                    \
               blocks_for(pairs), kBlock, smem, s,                             \
        x, w, bias, y, Ci, H, W, OH, OW, KH, KW, SH, SW, PH, PW, act,          \
        static_cast<uint32_t>(pairs), FastDiv(per_row), FastDiv(OH));          \
    return cudaGetLastError();                                                 \
  }
    PB2_STEM2(16)
    PB2_STEM2(32)
    PB2_STEM2(48)
#undef PB2_STEM2
  }
  if (Ci <= 4 && (Co == 16 || Co == 32 || Co == 48 || Co == 64) &&
      pixels < (1LL << 31)) {
#define PB2_STEM(co)                                                           \
  if (Co == co) {                                                              \
    launch_pdl(act == kActRelu ? stem_conv_kernel<co, kActRelu>                \
                               : stem_conv_kernel<co, -1>,                     \
               blocks_for(pixels), kBlock, smem, s,                            \
        x, w, bias, y, batch, Ci, H, W, OH, OW, KH, KW, SH, SW, PH, PW, act,   \
        static_cast<uint32_t>(pixels), FastDiv(OW), FastDiv(OH));              \
    return cudaGetLastError();                                                 \
  }
    PB2_STEM(16)
    PB2_STEM(32)
    PB2_STEM(48)
    PB2_STEM(64)
#undef PB2_STEM
  }
  const long long total = static_cast<long long>(batch) * OH * OW * (Co / 8);
  launch_pdl(direct_conv_kernel, blocks_for(total), kBlock, smem, s, x, w, bias, y, batch, Ci, H, W,
      Co, OH, OW, KH, KW, SH, SW, PH, PW, act);
  return cudaGetLastError();
}

cudaError_t pool_nhwc(const half *x, half *y, int batch, int C, int H, int W,
                      int OH, int OW, int KH, int KW, int SH, int SW, int PH,
                      int PW, bool maximum, cudaStream_t s) {
  if (C % 8 == 0 && al16(x) && al16(y) && PH == 0 && PW == 0 &&
      (OH - 1) * SH + KH <= H && (OW - 1) * SW + KW <= W) {
    const long long total = static_cast<long long>(batch) * OH * OW * (C / 8);
    if (!maximum && KH == 3 && KW == 2 && SH == 3 && SW == 2) {
      launch_pdl(pool_fixed_kernel<3, 2, 3, 2, false>, blocks_for(total), kBlock, 0, s, x, y, batch,
          C, H, W, OH, OW, FastDiv(static_cast<uint32_t>(C / 8)),
          FastDiv(static_cast<uint32_t>(OW)), FastDiv(static_cast<uint32_t>(OH)));
      return cudaGetLastError();
    }
    if (maximum && KH == 2 && KW == 2 && SH == 1 && SW == 1) {
      launch_pdl(pool_fixed_kernel<2, 2, 1, 1, true>, blocks_for(total), kBlock, 0, s, x, y, batch,
          C, H, W, OH, OW, FastDiv(static_cast<uint32_t>(C / 8)),
          FastDiv(static_cast<uint32_t>(OW)), FastDiv(static_cast<uint32_t>(OH)));
      return cudaGetLastError();
    }
  }
  if (C % 8 == 0 && al16(x) && al16(y)) {
    const long long total = static_cast<long long>(batch) * OH * OW * (C / 8);
    launch_pdl(pool_nhwc_vec_kernel, blocks_for(total), kBlock, 0, s, x, y, batch, C, H, W, OH, OW,
        KH, KW, SH, SW, PH, PW, maximum);
  } else {
    const long long total = static_cast<long long>(batch) * OH * OW * C;
    launch_pdl(pool_scalar_kernel, blocks_for(total), kBlock, 0, s, x, y, total, C, H, W, OH, OW,
        KH, KW, SH, SW, PH, PW, maximum, true);
  }
  return cudaGetLastError();
}

cudaError_t pool_nchw(const half *x, half *y, int planes, int H, int W, int OH,
                      int OW, int KH, int KW, int SH, int SW, int PH, int PW,
                      bool maximum, cudaStream_t s) {
  const long long total = static_cast<long long>(planes) * OH * OW;
  launch_pdl(pool_scalar_kernel, blocks_for(total), kBlock, 0, s, x, y, total, 1, H, W, OH, OW, KH,
      KW, SH, SW, PH, PW, maximum, false);
  return cudaGetLastError();
}

cudaError_t pad_nhwc(const half *x, half *y, int batch, int C, int H, int W,
                     int OH, int OW, int PH, int PW, cudaStream_t s) {
  const bool vec = C % 8 == 0 && al16(x) && al16(y);
  const long long total =
      static_cast<long long>(batch) * OH * OW * (vec ? C / 8 : C);
  launch_pdl(pad_kernel, blocks_for(total), kBlock, 0, s, x, y, total, C, H, W, OH, OW, PH, PW, vec);
  return cudaGetLastError();
}

cudaError_t pad_nchw(const half *x, half *y, int planes, int H, int W, int OH,
                     int OW, int PH, int PW, cudaStream_t s) {
  const long long total = static_cast<long long>(planes) * OH * OW;
  launch_pdl(pad_kernel, blocks_for(total), kBlock, 0, s, x, y, total, 1, H, W, OH, OW, PH, PW,
      false);
  return cudaGetLastError();
}

cudaError_t resize_nearest_nhwc(const half *x, const half *addend, half *y,
                                int batch, int C, int H, int W, int OH, int OW,
                                float sh, float sw, cudaStream_t s) {
  const bool vec =
      C % 8 == 0 && al16(x) && al16(y) && (!addend || al16(addend));
  const long long total =
      static_cast<long long>(batch) * OH * OW * (vec ? C / 8 : C);
  if (vec && total < (1LL << 31)) {
    launch_pdl(resize_nhwc_vec_kernel, blocks_for(total), kBlock, 0, s, x, addend, y,
        static_cast<uint32_t>(total), C, H, W, FastDiv(static_cast<uint32_t>(C / 8)),
        FastDiv(static_cast<uint32_t>(OW)), FastDiv(static_cast<uint32_t>(OH)), sh, sw);
    return cudaGetLastError();
  }
  launch_pdl(resize_nhwc_kernel, blocks_for(total), kBlock, 0, s, x, addend, y, total, C, H, W, OH,
      OW, sh, sw, vec);
  return cudaGetLastError();
}

cudaError_t upsample_concat_nhwc(const UpcatArgs &a, half *y, int batch, int OH, int OW,
                                 cudaStream_t s) {
  if (a.n < 1 || a.n > kUpcatMax || !al16(y))
    return cudaErrorInvalidValue;
  long long ctot = 0;
  for (int k = 0; k < a.n; ++k) {
    if (!a.src[k] || a.C[k] <= 0 || a.C[k] % 8 || !al16(a.src[k]) || a.H[k] <= 0 || a.W[k] <= 0 ||
        !(a.sh[k] > 0.f) || !(a.sw[k] > 0.f))
      return cudaErrorInvalidValue;
    ctot += a.C[k];
  }
  if (batch <= 0 || OH <= 0 || OW <= 0)
    return cudaSuccess;
  const long long total = static_cast<long long>(batch) * OH * OW * (ctot / 8);
  if (total >= (1LL << 31))
    return cudaErrorInvalidValue;
  launch_pdl(upsample_concat_kernel, blocks_for(total), kBlock, 0, s, a, y,
      static_cast<uint32_t>(total), FastDiv(static_cast<uint32_t>(ctot / 8)),
      FastDiv(static_cast<uint32_t>(OW)), FastDiv(static_cast<uint32_t>(OH)));
  return cudaGetLastError();
}

cudaError_t resize_nearest_nchw(const half *x, half *y, int planes, int H,
                                int W, int OH, int OW, float sh, float sw,
                                cudaStream_t s) {
  const long long total = static_cast<long long>(planes) * OH * OW;
  launch_pdl(resize_nchw_kernel, blocks_for(total), kBlock, 0, s, x, y, total, H, W, OH, OW, sh, sw);
  return cudaGetLastError();
}

cudaError_t concat_rows(const half *a, const half *b, half *y, long long rows,
                        int na, int nb, cudaStream_t s) {
  const bool vec = na % 8 == 0 && nb % 8 == 0 && al16(a) && al16(b) && al16(y);
  const int wa = vec ? na / 8 : na, wb = vec ? nb / 8 : nb;
  const long long total = rows * (wa + wb);
  launch_pdl(concat_kernel, blocks_for(total), kBlock, 0, s, a, b, y, total, wa, wb, vec);
  return cudaGetLastError();
}

cudaError_t transpose2d(const half *x, half *y, int batch, int rows, int cols,
                        cudaStream_t s) {
  if (batch <= 0 || rows <= 0 || cols <= 0)
    return cudaSuccess;
  dim3 grid((cols + 31) / 32, (rows + 31) / 32, batch);
  launch_pdl(transpose_kernel, grid, dim3(32, 8), 0, s, x, y, rows, cols);
  return cudaGetLastError();
}

cudaError_t gather(const half *x, half *y, long long n, const Gather &g,
                   cudaStream_t s) {
  if (n <= 0)
    return cudaSuccess;
  launch_pdl(gather_kernel, blocks_for(n), kBlock, 0, s, x, y, n, g);
  return cudaGetLastError();
}

cudaError_t binary(const half *a, const half *b, half *y, long long n,
                   const Gather &ga, const Gather &gb, int op,
                   cudaStream_t s) {
  if (n <= 0)
    return cudaSuccess;
  launch_pdl(binary_kernel, blocks_for(n), kBlock, 0, s, a, b, y, n, ga, gb, op);
  return cudaGetLastError();
}

cudaError_t binary_flat(const half *a, const half *b, half *y, long long n,
                        int ad, int am, int bd, int bm, int op,
                        cudaStream_t s) {
  if (n <= 0)
    return cudaSuccess;
  launch_pdl(binary_flat_kernel, blocks_for(n), kBlock, 0, s, a, b, y, n, ad, am, bd, bm, op);
  return cudaGetLastError();
}

cudaError_t unary(const half *x, half *y, long long n, int op, float alpha,
                  float beta, cudaStream_t s) {
  if (n <= 0)
    return cudaSuccess;
  launch_pdl(unary_kernel, blocks_for(n), kBlock, 0, s, x, y, n, op, alpha, beta);
  return cudaGetLastError();
}

cudaError_t copy_input_f32(const float *x, half *y, size_t valid, size_t total,
                           cudaStream_t s) {
  if (!total)
    return cudaSuccess;
  launch_pdl(copy_input_f32_kernel, blocks_for(static_cast<long long>(total)), kBlock, 0, s, x, y,
      valid, total);
  return cudaGetLastError();
}

cudaError_t copy_input_nhwc_f16(const half *x, half *y, int valid, int batch,
                                int C, int H, int W, cudaStream_t s) {
  const long long total = static_cast<long long>(batch) * C * H * W;
  if (total <= 0)
    return cudaSuccess;
  if (C == 1 || static_cast<long long>(H) * W == 1) {
    // One channel (or one pixel): NHWC and NCHW are the same layout, so the
    // valid images are one contiguous copy and the rest is zero.
    const size_t image = static_cast<size_t>(C) * H * W * sizeof(half);
    return stage_bytes(x, y, image * valid, image * batch, s);
  }
  launch_pdl(copy_input_nhwc_kernel, blocks_for(total), kBlock, 0, s, x, y, valid, total, C, H, W);
  return cudaGetLastError();
}

namespace {

__global__ void __launch_bounds__(kBlock)
    stage_bytes_kernel(const uint4 *__restrict__ x, uint4 *__restrict__ y, size_t valid16,
                       size_t total16) {
  pdl_begin();
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total16;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    y[i] = i < valid16 ? __ldg(x + i) : make_uint4(0, 0, 0, 0);
}

// Thread = 8 consecutive values (n % 8 == 0, 16-byte aligned) or one value.
template <bool VEC, bool F32>
__global__ void __launch_bounds__(kBlock)
    output_copy_kernel(const half *__restrict__ x, void *__restrict__ y, size_t n,
                       const int *__restrict__ err, int *__restrict__ err_host) {
  pdl_begin();
  if (blockIdx.x == 0 && threadIdx.x == 0 && err_host)
    *reinterpret_cast<volatile int *>(err_host) = *reinterpret_cast<const volatile int *>(err);
  const size_t step = static_cast<size_t>(gridDim.x) * blockDim.x;
  if constexpr (VEC) {
    const uint4 *xv = reinterpret_cast<const uint4 *>(x);
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n / 8; i += step) {
      Pack8 p;
      p.u = __ldg(xv + i);
      if constexpr (F32) {
        float4 *yv = reinterpret_cast<float4 *>(y) + 2 * i;
        const float2 a = __half22float2(p.h[0]), b = __half22float2(p.h[1]);
        const float2 c = __half22float2(p.h[2]), d = __half22float2(p.h[3]);
        yv[0] = make_float4(a.x, a.y, b.x, b.y);
        yv[1] = make_float4(c.x, c.y, d.x, d.y);
      } else {
        reinterpret_cast<uint4 *>(y)[i] = p.u;
      }
    }
  } else {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += step) {
      if constexpr (F32)
        reinterpret_cast<float *>(y)[i] = __half2float(x[i]);
      else
        reinterpret_cast<half *>(y)[i] = x[i];
    }
  }
}

// Grid-stride launches: a few CTAs per SM cover any size.
unsigned stride_blocks(size_t items) {
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  const size_t b = (items + kBlock - 1) / kBlock;
  return static_cast<unsigned>(b < 1 ? 1 : b > cap ? cap : b);
}

} // namespace

cudaError_t stage_bytes(const void *x, void *y, size_t valid, size_t total, cudaStream_t s) {
  if (!total)
    return cudaSuccess;
  if (valid > total)
    return cudaErrorInvalidValue;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | valid | total) & 15) == 0)
    return launch_pdl(stage_bytes_kernel, stride_blocks(total / 16), kBlock, 0, s,
                      static_cast<const uint4 *>(x), static_cast<uint4 *>(y), valid / 16, total / 16);
  cudaError_t e = valid ? cudaMemcpyAsync(y, x, valid, cudaMemcpyDeviceToDevice, s) : cudaSuccess;
  if (e == cudaSuccess && valid < total)
    e = cudaMemsetAsync(static_cast<char *>(y) + valid, 0, total - valid, s);
  return e;
}

cudaError_t output_copy(const half *x, void *y, size_t n, bool to_f32, const int *err, int *err_host,
                        cudaStream_t s) {
  const bool vec = n % 8 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  const unsigned blocks = stride_blocks(vec ? n / 8 : n);
  if (vec)
    return to_f32 ? launch_pdl(output_copy_kernel<true, true>, blocks, kBlock, 0, s, x, y, n, err, err_host)
                  : launch_pdl(output_copy_kernel<true, false>, blocks, kBlock, 0, s, x, y, n, err, err_host);
  return to_f32 ? launch_pdl(output_copy_kernel<false, true>, blocks, kBlock, 0, s, x, y, n, err, err_host)
                : launch_pdl(output_copy_kernel<false, false>, blocks, kBlock, 0, s, x, y, n, err, err_host);
}

cudaError_t half_to_float(const half *x, float *y, size_t n, cudaStream_t s) {
  if (!n)
    return cudaSuccess;
  launch_pdl(half_to_float_kernel, blocks_for(static_cast<long long>(n)), kBlock, 0, s, x, y, n);
  return cudaGetLastError();
}

} // namespace pb2
