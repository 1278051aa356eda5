// Fused depthwise-separable block: depthwise KxK (stride 1, same padding,
// + bias + activation) followed by a pointwise 1x1 GEMM (+ bias +
// activation), the depthwise output never leaving the SM.
//
// Replaces the reference's pair Runtime::conv (depthwise, native/src/
// compiled/runtime.cuh:668-765; its 5x5 goes to cuDNN) + Runtime::
// gemm_epilogue (runtime.cuh:514-646, cuBLASLt/CUTLASS) for BASELINE config 2
// (FP16 NHWC [16,48,320,64], dw 5x5 -> pw 64->128, folded BN + hardswish):
// unfused, the 31.5 MB depthwise output is written to HBM and read back.
//
// Tile: 2 output rows x 64 output columns = 128 pixels of one image, all 64
// channels. Per tile:
//  * warp 0 loads the input halo, (K+1) rows x (64+K-1) columns x 64
//    channels, as one 4-D TMA box (128-byte swizzled; pixels outside the
//    image zero-filled) into a 2-deep ring;
//  * warps 2-9 (256 threads, 4 pixels x 8 channels each) compute the
//    depthwise taps in the reference's order with one mixed-precision FMA per
//    multiply-add (rows outside the image skipped, as the reference and the
//    standalone depthwise kernels do: bit-identical to them), apply bias +
//    activation with the fp16 rounding of a stored tensor, and write the
//    fp16 result as the 128 x 64 K-major, 128-byte swizzled A operand of the
//    pointwise GEMM (double buffered);
//  * warp 1 issues the 4 tcgen05.mma (M 128, N Co, K 16) against the
//    resident pointwise filter into a double-buffered TMEM accumulator;
//  * warps 10-13 drain it (bias + activation, fp16 NHWC stores).
// One persistent CTA per SM; every wait is bounded.
#include "kernels.h"
#include "ptx.cuh"
#include <mutex>

namespace pb2 {
namespace {

constexpr int kDwThreads = 256;
constexpr int kDwpwThreads = 32 * 14; // producer, MMA, 8 depthwise, 4 epilogue warps
constexpr int kTileRows = 2, kTileCols = 64;

struct DwpwArgs {
  const half *wdw;   // [64][K][K]
  const half *bdw;   // [64] or null
  const half *bpw;   // [Co] or null
  half *y;           // [B][H][W][Co]
  int B, H, W, Co;
  int act_dw, act_pw;
  int tiles_w, tiles_h, tiles;
  uint32_t halo_bytes, halo_stride;
  int *err;
};

__device__ __forceinline__ void dwpw_fail(const DwpwArgs &g, volatile int *abort, int code) {
  *abort = 1;
  if (g.err)
    atomicCAS(g.err, 0, code);
}

template <int K, int CO, int ACT1, int ACT2>
__global__ void __launch_bounds__(kDwpwThreads, 1)
    dwpw_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW,
                const __grid_constant__ DwpwArgs g) {
  constexpr int P = K / 2;
  constexpr int HW = kTileCols + K - 1;    // halo columns
  constexpr int NCOL = 4 + K - 1;          // halo columns one thread reads per row
  constexpr uint32_t A_BYTES = 128 * 128;  // 128 pixels x 64 channels fp16
  constexpr uint32_t W_BYTES = CO * 128;   // pointwise filter, 128-byte rows
  constexpr int ACC = CO <= 64 ? 64 : CO <= 128 ? 128 : 256;
  constexpr uint32_t TMEM_COLS = 2 * ACC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *halo = smem;                           // [2][halo_stride]
  uint8_t *abuf = halo + 2 * g.halo_stride;       // [2][A_BYTES]
  uint8_t *wpw = abuf + 2 * A_BYTES;              // [CO][128 B]
  half *wdw = reinterpret_cast<half *>(wpw + ((W_BYTES + 1023) & ~1023u)); // [K*K][64]
  half *bdw = wdw + K * K * 64;                   // [64]
  half *bpw = bdw + 64;                           // [CO] pointwise bias (staged)
  uint64_t *bars = reinterpret_cast<uint64_t *>(bpw + CO);
  uint64_t *hfull = bars, *hempty = bars + 2, *afull = bars + 4, *aempty = bars + 6;
  uint64_t *tfull = bars + 8, *tempty = bars + 10, *wbar = bars + 12, *drain = bars + 13;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 14);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&hfull[i], 1);
      mbar_init(&hempty[i], kDwThreads);
      mbar_init(&afull[i], kDwThreads);
      mbar_init(&aempty[i], 1);
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(wbar, 1);
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  // First global-memory access below (programmatic dependent launch).
  pdl_wait();
  // Depthwise filter tap-major ([tap][channel]) and bias, staged once.
  for (int i = threadIdx.x; i < K * K * 64; i += blockDim.x) {
    const int tap = i >> 6, c = i & 63;
    wdw[i] = g.wdw[c * K * K + tap];
  }
  if (threadIdx.x < 64)
    bdw[threadIdx.x] = g.bdw ? g.bdw[threadIdx.x] : __float2half(0.f);
  for (int c = threadIdx.x; c < CO; c += blockDim.x)
    bpw[c] = g.bpw ? g.bpw[c] : __float2half(0.f);
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&mapX);
      prefetch_tensormap(&mapW);
      mbar_arrive_expect_tx(wbar, W_BYTES);
      tma_load_2d(wpw, &mapW, wbar, 0, 0);
      uint32_t issued = 0, issued_par = 0;
      int it = 0;
      for (int t = blockIdx.x; t < g.tiles; t += gridDim.x, ++it) {
        const int s = it & 1;
        const uint32_t par = (it >> 1) & 1;
        if (!mbar_wait(&hempty[s], par ^ 1, abort)) {
          dwpw_fail(g, abort, 31);
          break;
        }
        const int tw = t % g.tiles_w, rest = t / g.tiles_w;
        const int th = rest % g.tiles_h, n = rest / g.tiles_h;
        mbar_arrive_expect_tx(&hfull[s], g.halo_bytes);
        issued |= 1u << s;
        issued_par = (issued_par & ~(1u << s)) | (par << s);
        tma_load_4d(halo + s * g.halo_stride, &mapX, &hfull[s], 0, tw * kTileCols - P, th * kTileRows - P, n);
      }
      for (int s = 0; s < 2; ++s)
        if (issued & (1u << s)) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&hfull[s], (issued_par >> s) & 1u) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      const long long t0 = clock64();
      while (!mbar_try_wait(wbar, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(128, CO);
      const uint64_t bdesc = sdesc_k_sw128(smem_u32(wpw));
      bool ok = mbar_wait(wbar, 0, abort);
      if (!ok)
        dwpw_fail(g, abort, 32);
      int it = 0;
      for (int t = blockIdx.x; ok && t < g.tiles; t += gridDim.x, ++it) {
        const int a = it & 1;
        const uint32_t par = (it >> 1) & 1;
        if (!mbar_wait(&afull[a], par, abort) || !mbar_wait(&tempty[a], par ^ 1, abort)) {
          dwpw_fail(g, abort, 33);
          break;
        }
        tc_fence_after();
        const uint64_t adesc = sdesc_k_sw128(smem_u32(abuf + a * A_BYTES));
        const uint32_t d = tmem_base + a * ACC;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, k != 0);
        umma_commit(&aempty[a]);
        umma_commit(&tfull[a]);
      }
      umma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else if (warp < 10) {
    // Depthwise: thread = 8 channels (chunk j) x 4 consecutive pixels of
    // one of the tile's two rows.
    const int d = threadIdx.x - 64;
    const int j = d & 7, r = (d >> 3) & 1, px0 = (d >> 4) * 4;
    float bv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e)
      bv[e] = __half2float(bdw[j * 8 + e]);
    const bool has_bias = g.bdw != nullptr;
    const uint32_t wdw_s = smem_u32(wdw);
    int it = 0;
    for (int t = blockIdx.x; t < g.tiles; t += gridDim.x, ++it) {
      const int s = it & 1, a = it & 1;
      const uint32_t par = (it >> 1) & 1;
      if (!mbar_wait(&hfull[s], par, abort) || !mbar_wait(&aempty[a], par ^ 1, abort)) {
        dwpw_fail(g, abort, 34);
        break;
      }
      const int rest = t / g.tiles_w;
      const int th = rest % g.tiles_h;
      const int oy = th * kTileRows + r; // this thread's output row
      const uint32_t hbase = smem_u32(halo + s * g.halo_stride);
      float acc[4][8];
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int e = 0; e < 8; ++e)
          acc[p][e] = 0.f;
#pragma unroll
      for (int kh = 0; kh < K; ++kh) {
        const int iy = oy - P + kh;
        if (iy < 0 || iy >= g.H)
          continue; // rows outside the image are skipped
        uint4 strip[NCOL];
#pragma unroll
        for (int q = 0; q < NCOL; ++q) {
          const uint32_t pix = static_cast<uint32_t>((r + kh) * HW + px0 + q);
          strip[q] = lds_v4(hbase + pix * 128u + ((static_cast<uint32_t>(j) ^ (pix & 7u)) << 4));
        }
#pragma unroll
        for (int kw = 0; kw < K; ++kw) {
          const uint4 wt = lds_v4(wdw_s + static_cast<uint32_t>(((kh * K + kw) * 64 + j * 8) * 2));
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint4 xv = strip[p + kw];
            fma2_h(acc[p][0], acc[p][1], xv.x, wt.x);
            fma2_h(acc[p][2], acc[p][3], xv.y, wt.y);
            fma2_h(acc[p][4], acc[p][5], xv.z, wt.z);
            fma2_h(acc[p][6], acc[p][7], xv.w, wt.w);
          }
        }
      }
      // The halo stage is no longer read by this thread.
      mbar_arrive(&hempty[s]);
      const uint32_t abase = smem_u32(abuf + a * A_BYTES);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v0 = round_half(acc[p][2 * e]);
          float v1 = round_half(acc[p][2 * e + 1]);
          if (has_bias) {
            v0 = act_t<ACT1>(v0 + bv[2 * e], g.act_dw);
            v1 = act_t<ACT1>(v1 + bv[2 * e + 1], g.act_dw);
          }
          const half2 h = __floats2half2_rn(v0, v1);
          o[e] = *reinterpret_cast<const uint32_t *>(&h);
        }
        const uint32_t m = static_cast<uint32_t>(r * kTileCols + px0 + p); // A row
        sts_v4(abase + m * 128u + ((static_cast<uint32_t>(j) ^ (m & 7u)) << 4), make_uint4(o[0], o[1], o[2], o[3]));
      }
      fence_async_smem(); // generic-proxy writes -> tensor-core reads
      mbar_arrive(&afull[a]);
    }
  } else {
    // Epilogue: warp w drains TMEM lane quarter w % 4 (tile row m).
    const int q = warp & 3;
    const int m = q * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < g.tiles; t += gridDim.x, ++it) {
      const int a = it & 1;
      if (!mbar_wait(&tfull[a], (it >> 1) & 1, abort)) {
        dwpw_fail(g, abort, 35);
        break;
      }
      tc_fence_after();
      const int tw = t % g.tiles_w, rest = t / g.tiles_w;
      const int th = rest % g.tiles_h, n = rest / g.tiles_h;
      const int oy = th * kTileRows + m / kTileCols, ox = tw * kTileCols + m % kTileCols;
      const bool valid = oy < g.H && ox < g.W;
      half *dst = g.y + ((static_cast<long long>(n) * g.H + oy) * g.W + ox) * CO;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + a * ACC;
#pragma unroll
      for (int c0 = 0; c0 < CO; c0 += 64) {
        uint32_t rr[64];
#pragma unroll
        for (int c = 0; c < 64; c += 16)
          tmem_ld16(taddr + c0 + c, *reinterpret_cast<uint32_t(*)[16]>(rr + c));
        tmem_ld_wait();
        if (valid) {
#pragma unroll
          for (int h = 0; h < 8; ++h) {
            const int cc = c0 + 8 * h;
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              v[e] = round_half(__uint_as_float(rr[8 * h + e]));
            if (g.bpw) {
              const uint4 bb = lds_v4(smem_u32(bpw + cc));
              const half2 *bh = reinterpret_cast<const half2 *>(&bb);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(bh[e]);
                v[2 * e] += f.x;
                v[2 * e + 1] += f.y;
              }
            }
            uint4 o;
            half2 *oh2 = reinterpret_cast<half2 *>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              oh2[e] = __floats2half2_rn(act_t<ACT2>(v[2 * e], g.act_pw), act_t<ACT2>(v[2 * e + 1], g.act_pw));
            *reinterpret_cast<uint4 *>(dst + cc) = o;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int K, int CO, int ACT1, int ACT2>
cudaError_t launch_dwpw(const CUtensorMap &mx, const CUtensorMap &mw, const DwpwArgs &g, cudaStream_t s) {
  auto kernel = dwpw_kernel<K, CO, ACT1, ACT2>;
  const size_t smem = 1024 + 2 * size_t(g.halo_stride) + 2 * 16384 + ((CO * 128 + 1023) & ~1023) + K * K * 128 +
                      128 + CO * 2 + 256;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
  });
  if (attr != cudaSuccess)
    return attr;
  if (smem > 232448)
    return cudaErrorNotSupported;
  const int grid = g.tiles < sm_count() ? g.tiles : sm_count();
  launch_pdl(kernel, grid, kDwpwThreads, smem, s, mx, mw, g);
  return cudaGetLastError();
}

template <int K, int CO>
cudaError_t dispatch_dwpw_act(const CUtensorMap &mx, const CUtensorMap &mw, const DwpwArgs &g, cudaStream_t s) {
  if (g.act_dw == kActHardSwish && g.act_pw == kActHardSwish)
    return launch_dwpw<K, CO, kActHardSwish, kActHardSwish>(mx, mw, g, s);
  if (g.act_dw == kActRelu && g.act_pw == kActRelu)
    return launch_dwpw<K, CO, kActRelu, kActRelu>(mx, mw, g, s);
  return launch_dwpw<K, CO, -1, -1>(mx, mw, g, s);
}

} // namespace

bool dwpw_supported(int C, int K, int Co) {
  return C == 64 && (K == 3 || K == 5) && (Co == 64 || Co == 128);
}

cudaError_t dwpw_block(const half *x, const half *wdw, const half *bdw, int act_dw, const half *wpw,
                       const half *bpw, int act_pw, half *y, int B, int H, int W, int C, int K, int Co,
                       cudaStream_t stream) {
  if (B <= 0 || H <= 0 || W <= 0)
    return cudaSuccess;
  if (!dwpw_supported(C, K, Co))
    return cudaErrorNotSupported;
  auto mis = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (mis(x) || mis(wpw) || mis(y) || (bpw && mis(bpw)) || !wdw)
    return cudaErrorInvalidValue;
  DwpwArgs g{};
  g.wdw = wdw;
  g.bdw = bdw;
  g.bpw = bpw;
  g.y = y;
  g.B = B;
  g.H = H;
  g.W = W;
  g.Co = Co;
  g.act_dw = act_dw;
  g.act_pw = act_pw;
  g.tiles_w = (W + kTileCols - 1) / kTileCols;
  g.tiles_h = (H + kTileRows - 1) / kTileRows;
  const long long tiles = static_cast<long long>(B) * g.tiles_w * g.tiles_h;
  if (tiles > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  g.tiles = static_cast<int>(tiles);
  const int hw = kTileCols + K - 1, hr = kTileRows + K - 1;
  g.halo_bytes = static_cast<uint32_t>(hr * hw * 128);
  g.halo_stride = (g.halo_bytes + 1023) & ~1023u;
  g.err = device_error_word();
  CUtensorMap mx, mw;
  cuuint64_t dx[4] = {64, static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t sx[3] = {128, static_cast<cuuint64_t>(W) * 128, static_cast<cuuint64_t>(H) * W * 128};
  cuuint32_t bx[4] = {64, static_cast<cuuint32_t>(hw), static_cast<cuuint32_t>(hr), 1};
  cuuint64_t dw[2] = {64, static_cast<cuuint64_t>(Co)};
  cuuint64_t sw[1] = {128};
  cuuint32_t bw[2] = {64, static_cast<cuuint32_t>(Co)};
  if (!encode_fp16_map(&mx, x, 4, dx, sx, bx, true) || !encode_fp16_map(&mw, wpw, 2, dw, sw, bw, true))
    return cudaErrorNotSupported;
  if (K == 5)
    return Co == 128 ? dispatch_dwpw_act<5, 128>(mx, mw, g, stream) : dispatch_dwpw_act<5, 64>(mx, mw, g, stream);
  return Co == 128 ? dispatch_dwpw_act<3, 128>(mx, mw, g, stream) : dispatch_dwpw_act<3, 64>(mx, mw, g, stream);
}

} // namespace pb2
