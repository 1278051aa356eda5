// Stem convolution on the tensor cores: 3x3, stride 2, padding 1, three input
// channels (the first layer of the recognizer and the detector), replacing
// the reference's cuDNN convolution (native/src/compiled/runtime.cuh:
// 766-815) and this library's SIMT stem kernel.
//
// With Ci = 3 the contraction is only K = 27 deep, so there is nothing to
// stage per tap; instead SIMT warps build the im2col rows themselves from
// input rows held in shared memory and the tensor core does the 27 x Co
// product:
//  * work unit = R output rows of one image; warp 0 brings the unit's 2R+1
//    input rows into shared memory with one cp.async.bulk copy (rows of an
//    NHWC image are contiguous), two units in flight;
//  * two groups of four builder warps take alternate 128-pixel tiles; a
//    thread writes one A row (output pixel): K = (kh, kw, ci) for 27 columns
//    + 5 zero columns, in the canonical no-swizzle K-major layout (8-column
//    groups as planes of 128 rows x 16 bytes). Each window row of the pixel
//    is 9 consecutive halves starting 2 bytes into a 4-byte word, so it is
//    read as 5 aligned words and realigned with byte permutes; columns and
//    rows outside the image are zero;
//  * warp 1 issues the two K = 16 UMMAs against the resident filter
//    (Co rows x 32 columns, same layout) into a double-buffered TMEM
//    accumulator;
//  * four warps drain it with the fused bias + activation into a staging
//    tile and one thread writes the tile's 128 NHWC pixels (consecutive in
//    memory) with a single bulk copy.
// The sums run over (kh, kw, ci) in fp32 inside the tensor core, in its own
// order (the SIMT kernel summed sequentially): results agree to fp32
// rounding, not bit for bit. Every wait is bounded.
#include "kernels.h"
#include "ptx.cuh"
#include <mutex>

namespace pb2 {
namespace {

constexpr int kStemThreads = 32 * 14;
constexpr int kStemK = 32;           // 27 taps x channels + 5 zeros
constexpr uint32_t kAPlane = 128 * 16;        // one 8-column group of 128 rows
constexpr uint32_t kABytes = 4 * kAPlane;     // 128 rows x 32 columns

struct StemArgs {
  const half *x;     // [B][H][W][3]
  const half *w;     // [Co][3][3][3]
  const half *bias;  // [Co] or null
  half *y;           // [B][OH][OW][Co]
  int B, H, W, OH, OW, Co;
  int R;             // output rows per unit
  int units_per_image, units;
  int tiles;         // 128-pixel tiles per unit
  FastDiv ow_div;    // q -> (q / OW)
  uint32_t in_stride; // bytes per input buffer (2R+1 rows, 1024-aligned)
  int act;
  int *err;
};

__device__ __forceinline__ uint64_t sdesc_none(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

__device__ __forceinline__ void stem_fail(const StemArgs &g, volatile int *abort, int code) {
  *abort = 1;
  if (g.err)
    atomicCAS(g.err, 0, code);
}

// Bias + activation of two fp32 accumulators -> two fp16 outputs. The
// accumulator is rounded to fp16 first (the reference's convolution writes
// fp16 before its bias add). For none/ReLU the add runs as one fp16x2 add:
// a correctly rounded fp16 sum equals the fp32 sum rounded to fp16, since
// fp32 carries 24 >= 2 * 11 + 2 bits (Figueroa, "When is double rounding
// innocuous?", SIGNUM 1995), and ReLU commutes with rounding.
template <int ACT>
__device__ __forceinline__ uint32_t stem_out2(uint32_t a0, uint32_t a1, uint32_t bias2, int act) {
  if constexpr (ACT == kActNone || ACT == kActRelu) {
    __half2 h = __floats2half2_rn(__uint_as_float(a0), __uint_as_float(a1));
    h = __hadd2(h, *reinterpret_cast<const __half2 *>(&bias2));
    if constexpr (ACT == kActRelu)
      h = __hmax2(h, __float2half2_rn(0.f));
    return *reinterpret_cast<uint32_t *>(&h);
  } else {
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&bias2));
    const float v0 = act_t<ACT>(round_half(__uint_as_float(a0)) + b.x, act);
    const float v1 = act_t<ACT>(round_half(__uint_as_float(a1)) + b.y, act);
    const __half2 h = __floats2half2_rn(v0, v1);
    return *reinterpret_cast<const uint32_t *>(&h);
  }
}

template <int CO, int ACT>
__global__ void __launch_bounds__(kStemThreads, 1) stem_tc_kernel(const __grid_constant__ StemArgs g) {
  constexpr int ACC = CO <= 32 ? 32 : 64;
  constexpr uint32_t TMEM_COLS = 2 * ACC;
  constexpr uint32_t B_PLANE = CO * 16;
  constexpr uint32_t STAGE = 128 * CO * 2;       // one output tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *inb = smem;                             // [2][in_stride] input rows
  uint8_t *abuf = inb + 2 * g.in_stride;           // [2][kABytes]
  uint8_t *stage = abuf + 2 * kABytes;             // [2][STAGE]
  uint8_t *bbuf = stage + 2 * STAGE;               // [4][CO][16 B]
  uint8_t *bias_s = bbuf + 4 * B_PLANE;            // [CO] halves (128 B)
  uint64_t *bars = reinterpret_cast<uint64_t *>(bias_s + 128);
  uint64_t *ifull = bars, *iempty = bars + 2, *afull = bars + 4, *aempty = bars + 6;
  uint64_t *tfull = bars + 8, *tempty = bars + 10, *sfull = bars + 12, *sfree = bars + 14, *drain = bars + 16;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 17);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ifull[i], 1);
      mbar_init(&iempty[i], 256);
      mbar_init(&afull[i], 128);
      mbar_init(&aempty[i], 1);
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
      mbar_init(&sfull[i], 128);
      mbar_init(&sfree[i], 1);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  // First global-memory access below (programmatic dependent launch).
  pdl_wait();
  // Filter [CO][27] -> 4 planes of [CO][8] halves (columns 27..31 zero).
  for (int i = threadIdx.x; i < CO * kStemK; i += blockDim.x) {
    const int n = i / kStemK, k = i - n * kStemK;
    const half v = k < 27 ? g.w[n * 27 + k] : __float2half(0.f);
    reinterpret_cast<half *>(bbuf + (k >> 3) * B_PLANE + n * 16)[k & 7] = v;
  }
  if (threadIdx.x < CO)
    reinterpret_cast<half *>(bias_s)[threadIdx.x] = g.bias ? g.bias[threadIdx.x] : __float2half(0.f);
  fence_async_smem();
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const long long row_bytes = static_cast<long long>(g.W) * 6;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t issued = 0, issued_par = 0;
      int it = 0;
      for (int u = blockIdx.x; u < g.units; u += gridDim.x, ++it) {
        const int s = it & 1;
        const uint32_t par = (it >> 1) & 1;
        if (!mbar_wait(&iempty[s], par ^ 1, abort)) {
          stem_fail(g, abort, 41);
          break;
        }
        const int n = u / g.units_per_image, oy0 = (u - n * g.units_per_image) * g.R;
        // input rows 2*oy0 - 1 .. 2*(oy0 + R - 1) + 1, clipped to the image;
        // buffer row 0 is input row 2*oy0 - 1
        const int r_lo = max(0, 2 * oy0 - 1), r_hi = min(g.H - 1, 2 * (oy0 + g.R - 1) + 1);
        const uint32_t bytes = static_cast<uint32_t>((r_hi - r_lo + 1) * row_bytes);
        const int skip = r_lo - (2 * oy0 - 1); // 1 for the top unit
        mbar_arrive_expect_tx(&ifull[s], bytes);
        bulk_load(inb + s * g.in_stride + skip * row_bytes,
                  reinterpret_cast<const uint8_t *>(g.x) + (static_cast<long long>(n) * g.H + r_lo) * row_bytes, bytes,
                  &ifull[s]);
        issued |= 1u << s;
        issued_par = (issued_par & ~(1u << s)) | (par << s);
      }
      for (int s = 0; s < 2; ++s)
        if (issued & (1u << s)) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&ifull[s], (issued_par >> s) & 1u) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(128, CO);
      const uint64_t bdesc = sdesc_none(smem_u32(bbuf), B_PLANE, 128);
      int tc = 0; // tiles issued
      bool ok = true;
      for (int u = blockIdx.x; ok && u < g.units; u += gridDim.x) {
        for (int t = 0; t < g.tiles; ++t, ++tc) {
          const int a = tc & 1;
          const uint32_t par = (tc >> 1) & 1;
          if (!mbar_wait(&afull[a], par, abort) || !mbar_wait(&tempty[a], par ^ 1, abort)) {
            stem_fail(g, abort, 42);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sdesc_none(smem_u32(abuf + a * kABytes), kAPlane, 128);
          const uint32_t d = tmem_base + a * ACC;
          // K step k covers planes 2k, 2k+1 (LBO = plane stride)
          umma_f16(d, adesc, bdesc, idesc, 0);
          umma_f16(d, adesc + ((2 * kAPlane) >> 4), bdesc + ((2 * B_PLANE) >> 4), idesc, 1);
          umma_commit(&aempty[a]);
          umma_commit(&tfull[a]);
        }
      }
      umma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else if (warp < 10) {
    // Builders: group grp (warps 2-5 or 6-9) builds the tiles with
    // tc % 2 == grp into A buffer grp; thread = A row m.
    const int grp = (warp - 2) >> 2;
    const int m = threadIdx.x - 64 - grp * 128;
    const uint32_t rowb = static_cast<uint32_t>(g.W * 6);
    const uint32_t arow = smem_u32(abuf + grp * kABytes) + m * 16;
    int it = 0, tc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < g.units; u += gridDim.x, ++it) {
      const int s = it & 1;
      if (!mbar_wait(&ifull[s], (it >> 1) & 1, abort)) {
        stem_fail(g, abort, 43);
        break;
      }
      const int n = u / g.units_per_image, oy0 = (u - n * g.units_per_image) * g.R;
      const int rows_here = min(g.R, g.OH - oy0);
      const uint32_t in_s = smem_u32(inb + s * g.in_stride);
      for (int t = 0; t < g.tiles; ++t, ++tc) {
        if ((tc & 1) != grp)
          continue;
        if (!mbar_wait(&aempty[grp], ((tc >> 1) & 1) ^ 1, abort)) {
          stem_fail(g, abort, 44);
          ok = false;
          break;
        }
        const int q = t * 128 + m; // pixel of the unit
        const int oyl = static_cast<int>(g.ow_div.div(static_cast<uint32_t>(q))), ox = q - oyl * g.OW;
        uint32_t X[3][5];
#pragma unroll
        for (int kh = 0; kh < 3; ++kh)
#pragma unroll
          for (int a = 0; a < 5; ++a)
            X[kh][a] = 0u;
        if (oyl < rows_here) {
          // window row kh = buffer row 2*oyl + kh, columns 2*ox-1 .. 2*ox+1:
          // bytes [12*ox - 6, 12*ox + 12) of the row, read as the 5 words
          // from 12*ox - 8 (word a holds window halves 2a-1 and 2a)
          const bool left = ox > 0, right = 2 * ox + 1 < g.W;
          const uint32_t base = in_s + 2 * oyl * rowb + 12 * ox - 8;
          const int iy0 = 2 * (oy0 + oyl) - 1;
#pragma unroll
          for (int kh = 0; kh < 3; ++kh) {
            const int iy = iy0 + kh;
            if (iy >= 0 && iy < g.H) {
              const uint32_t ad = base + kh * rowb;
              if (left) {
                X[kh][0] = lds_u32(ad);
                X[kh][1] = lds_u32(ad + 4);
              }
              X[kh][2] = lds_u32(ad + 8);
              X[kh][3] = lds_u32(ad + 12);
              if (right)
                X[kh][4] = lds_u32(ad + 16);
              else
                X[kh][3] &= 0xFFFFu;
            }
          }
        }
        // K sequence: row 0 halves 0..8, row 1 halves 0..8, row 2 halves
        // 0..8, 5 zeros; word j = (K 2j, K 2j+1)
        uint32_t P[16];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          P[a] = __byte_perm(X[0][a], X[0][a + 1], 0x5432);
          P[9 + a] = __byte_perm(X[2][a], X[2][a + 1], 0x5432);
        }
        P[4] = __byte_perm(X[0][4], X[1][0], 0x7632);
        P[5] = X[1][1];
        P[6] = X[1][2];
        P[7] = X[1][3];
        P[8] = X[1][4];
        P[13] = X[2][4] >> 16;
        P[14] = 0u;
        P[15] = 0u;
#pragma unroll
        for (int pl = 0; pl < 4; ++pl)
          sts_v4(arow + pl * kAPlane, make_uint4(P[4 * pl], P[4 * pl + 1], P[4 * pl + 2], P[4 * pl + 3]));
        fence_async_smem();
        mbar_arrive(&afull[grp]);
      }
      mbar_arrive(&iempty[s]);
    }
  } else {
    // Epilogue: warp w drains TMEM lane quarter w % 4 (tile row m) into the
    // staging tile; thread 0 of warp 10 stores it.
    const int qd = warp & 3;
    const int m = qd * 32 + lane;
    const bool issuer = threadIdx.x == 320;
    const uint32_t bias_a = smem_u32(bias_s);
    int tc = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < g.units; u += gridDim.x) {
      const int n = u / g.units_per_image, oy0 = (u - n * g.units_per_image) * g.R;
      const int upix = min(g.R, g.OH - oy0) * g.OW;
      half *ybase = g.y + (static_cast<long long>(n) * g.OH + oy0) * g.OW * CO;
      for (int t = 0; t < g.tiles; ++t, ++tc) {
        const int a = tc & 1;
        if (!mbar_wait(&tfull[a], (tc >> 1) & 1, abort)) {
          stem_fail(g, abort, 45);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(qd * 32) << 16) + a * ACC;
        uint32_t r[CO];
#pragma unroll
        for (int c = 0; c < CO; c += 16)
          tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&tempty[a]);
        if (!mbar_wait(&sfree[a], ((tc >> 1) & 1) ^ 1, abort)) {
          stem_fail(g, abort, 46);
          ok = false;
          break;
        }
        const uint32_t srow = smem_u32(stage + a * STAGE) + m * (CO * 2);
#pragma unroll
        for (int h = 0; h < CO / 8; ++h) {
          const uint4 bb = lds_v4(bias_a + 16 * h);
          uint4 o;
          o.x = stem_out2<ACT>(r[8 * h + 0], r[8 * h + 1], bb.x, g.act);
          o.y = stem_out2<ACT>(r[8 * h + 2], r[8 * h + 3], bb.y, g.act);
          o.z = stem_out2<ACT>(r[8 * h + 4], r[8 * h + 5], bb.z, g.act);
          o.w = stem_out2<ACT>(r[8 * h + 6], r[8 * h + 7], bb.w, g.act);
          sts_v4(srow + 16 * h, o);
        }
        fence_async_smem();
        mbar_arrive(&sfull[a]);
        if (issuer) {
          if (!mbar_wait(&sfull[a], (tc >> 1) & 1, abort)) {
            stem_fail(g, abort, 47);
            ok = false;
            break;
          }
          // pixels of the tile inside the unit: none for the trailing tiles
          // of a short last unit
          const int npix = min(128, upix - t * 128);
          if (npix > 0) {
            bulk_store(ybase + static_cast<long long>(t) * 128 * CO, smem_u32(stage + a * STAGE),
                       static_cast<uint32_t>(npix * CO * 2));
            bulk_commit();
            // the previous tile's store has left its staging slot
            bulk_wait_read<1>();
          } else {
            bulk_wait_read<0>();
          }
          if (tc > 0)
            mbar_arrive(&sfree[a ^ 1]);
        }
      }
    }
    if (issuer)
      bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int CO, int ACT>
cudaError_t launch_stem(const StemArgs &g, size_t smem, cudaStream_t s) {
  auto kernel = stem_tc_kernel<CO, ACT>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
  });
  if (attr != cudaSuccess)
    return attr;
  const int grid = g.units < sm_count() ? g.units : sm_count();
  launch_pdl(kernel, grid, kStemThreads, smem, s, g);
  return cudaGetLastError();
}

template <int CO>
cudaError_t dispatch_stem_act(const StemArgs &g, size_t smem, cudaStream_t s) {
  return g.act == kActRelu ? launch_stem<CO, kActRelu>(g, smem, s) : launch_stem<CO, -1>(g, smem, s);
}

} // namespace

cudaError_t stem_conv_tc(const half *x, const half *w, const half *bias, half *y, int B, int H, int W, int Co,
                         int act, cudaStream_t s) {
  if (B <= 0 || H <= 0 || W <= 0)
    return cudaSuccess;
  const long long row_bytes = static_cast<long long>(W) * 6;
  if ((Co != 16 && Co != 32 && Co != 48 && Co != 64) || row_bytes % 16 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 15) || (bias && (reinterpret_cast<uintptr_t>(bias) & 15)))
    return cudaErrorNotSupported;
  StemArgs g{};
  g.x = x;
  g.w = w;
  g.bias = bias;
  g.y = y;
  g.B = B;
  g.H = H;
  g.W = W;
  g.OH = (H + 1) / 2;
  g.OW = (W + 1) / 2;
  g.Co = Co;
  g.act = act;
  g.err = device_error_word();
  // Output rows per unit: the largest count (at most 16) whose two input
  // buffers (2R+1 rows each) fit the budget, preferring a divisor of the
  // output height (no partial last unit); tiles per unit follow.
  const size_t fixed = 1024 + 2 * kABytes + 2 * size_t(128) * Co * 2 + 4 * Co * 16 + 128 + 256;
  int rmax = 16;
  while (rmax > 1 && fixed + 2 * (((2 * rmax + 1) * row_bytes + 1023) / 1024 * 1024) > 232448)
    --rmax;
  if (rmax > g.OH)
    rmax = g.OH;
  int R = rmax;
  for (int r = rmax; r >= (rmax + 1) / 2; --r)
    if (g.OH % r == 0) {
      R = r;
      break;
    }
  g.R = R;
  g.in_stride = static_cast<uint32_t>(((2 * R + 1) * row_bytes + 1023) / 1024 * 1024);
  const size_t smem = fixed + 2 * size_t(g.in_stride);
  if (smem > 232448 || (2 * R + 1) * row_bytes >= (1LL << 20))
    return cudaErrorNotSupported;
  g.units_per_image = (g.OH + R - 1) / R;
  const long long units = static_cast<long long>(B) * g.units_per_image;
  if (units > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  g.units = static_cast<int>(units);
  g.tiles = (R * g.OW + 127) / 128;
  g.ow_div = FastDiv(static_cast<uint32_t>(g.OW));
  switch (Co) {
  case 16:
    return dispatch_stem_act<16>(g, smem, s);
  case 32:
    return dispatch_stem_act<32>(g, smem, s);
  case 48:
    return dispatch_stem_act<48>(g, smem, s);
  default:
    return dispatch_stem_act<64>(g, smem, s);
  }
}

} // namespace pb2
