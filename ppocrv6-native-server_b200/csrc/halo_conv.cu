// Stride-1 3x3 dense convolution with few input channels (Ci = 16..64) on
// tcgen05, staging every input pixel in shared memory once per slab of
// output rows instead of once per filter tap.
//
// Replaces, for the HGNet stem / stage-1 layers (3x3, Ci = 48 at 24x160 and
// 12x80 in the recognizer; 480^2 and 240^2 in the detector), the reference's
// cuDNN dense convolution (native/src/compiled/runtime.cuh:766-815). The
// generic implicit GEMM in tc_gemm.cu loads one 128-byte channel block per
// pixel per tap: nine loads of every input pixel, which left these layers
// bound by L2->SM traffic and TMA issue.
//
// Layout: a slab is R output rows x Wt output columns of one image. Its
// input halo, (R + 2) rows x Wp = Wt + 2 columns, is one 4-D TMA box of 64
// channels per pixel, 128-byte swizzled: pixel p of the halo is the 128-byte
// row p of the slab (channels past Ci and pixels outside the image are
// zero-filled, which is the convolution's zero padding). Output pixels are
// enumerated "padded-flat", q = i * Wp + j (j >= Wt are discarded), so the
// A operand of filter tap (kh, kw) for the outputs [q0, q0 + 128) is the run
// of halo rows starting at q0 + kh * Wp + kw: a K-major SW128 UMMA
// descriptor whose start address moves by whole 128-byte rows. The
// hardware applies the 128-byte swizzle to absolute shared-memory address
// bits, the same rule TMA used when writing the slab, so any row offset
// addresses the right chunks (measured on B200 with shifted starts of 1, 3,
// 7 and 9 rows; the descriptor's base-offset field stays 0). K steps of 16
// channels move the start by 32 bytes inside the row.
//
// The filter ([Co][3][3][Ci]) of one N tile is resident in shared memory for
// the whole kernel: one 128-byte swizzled block of BN rows per tap.
//
// One persistent CTA per SM: warp 0 issues the TMA loads (filter once, then
// slabs into an NBUF-deep ring), warp 1 issues tcgen05.mma, warps 2-5 drain
// the accumulators (fused bias + activation, FP16 NHWC stores of the valid
// pixels). The NT 128-row tiles of a slab are computed together, their MMAs
// interleaved (tile 0, tile 1, ... for each tap and K step): consecutive
// MMAs into one accumulator depend on each other, and with N = 48-64 one
// MMA's math is shorter than that dependency, so a single tile's chain ran
// at a quarter of the tensor rate (measured). Accumulator sets are double
// buffered per slab (2 x NT x 64 TMEM columns). Every wait is bounded.
#include "kernels.h"
#include "ptx.cuh"
#include <mutex>

namespace pb2 {
namespace {

constexpr int kHaloThreads = 192;
constexpr int kMaxBufs = 4;
constexpr size_t kSmemLimit = 232448; // 227 KB of dynamic shared memory

struct HaloArgs {
  int OH, OW, batch;
  int R, Wt, Wp;       // slab: output rows, output columns, halo row pitch
  int row_blocks, col_blocks, slabs;
  int ntiles;          // N tiles of BN columns (CTA c serves N tile c % ntiles)
  int tiles;           // 128-row M tiles per slab (NT, the kernel's template argument)
  int ks;              // K = 16 steps per tap (Ci / 16)
  int nbuf;            // slab ring depth
  uint32_t slab_bytes; // (R + 2) * Wp * 128
  uint32_t slab_stride;
  uint32_t w_bytes;    // 9 * BN * 128
  uint32_t slack;      // bytes after the ring read by the last slab's last tile
  int Co, ldo;
  const half *bias;
  half *out;
  int act;
  int *err;
};

__device__ __forceinline__ void halo_fail(const HaloArgs &g, volatile int *abort, int code) {
  *abort = 1;
  if (g.err)
    atomicCAS(g.err, 0, code);
}
__device__ __forceinline__ void halo_fail(int *err, volatile int *abort, int code) {
  *abort = 1;
  if (err)
    atomicCAS(err, 0, code);
}

// TMEM columns for one accumulator of BN columns.
template <int BN> constexpr int acc_cols() { return BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256; }

// Epilogue of one 128-row accumulator: TMEM lane = padded-flat output
// index qrow (row i = qrow / wp, column j); rows past the slab, columns past
// Wt and pixels outside the image are not stored. Round to fp16, + bias,
// activation, 16-byte NHWC stores of up to BN columns from n0.
template <int BN, int ACT>
__device__ __forceinline__ void halo_drain_tile(uint32_t taddr, int qrow, int wp, int R, int Wt, int rb, int cb,
                                                int n, int OH, int OW, int ldo, int n0, int Co, const half *bias,
                                                half *out, int act) {
  const int i = qrow / wp, j = qrow - i * wp;
  const int oh = rb * R + i, ow = cb * Wt + j;
  const bool valid = i < R && j < Wt && oh < OH && ow < OW;
  half *dst = out + ((static_cast<long long>(n) * OH + oh) * OW + ow) * ldo;
  // Up to 64 columns per TMEM round trip: all loads, then one wait.
#pragma unroll
  for (int c0 = 0; c0 < BN; c0 += 64) {
    constexpr int kMax = BN < 64 ? BN : 64;
    uint32_t r[kMax];
#pragma unroll
    for (int c = 0; c < kMax; c += 16)
      tmem_ld16(taddr + c0 + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
    tmem_ld_wait();
    if (valid) {
#pragma unroll
      for (int h = 0; h < kMax / 8; ++h) {
        const int cc = n0 + c0 + 8 * h;
        if (cc < Co) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            v[e] = round_half(__uint_as_float(r[8 * h + e]));
          if (bias) {
            const uint4 bb = __ldg(reinterpret_cast<const uint4 *>(bias + cc));
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
            oh2[e] = __floats2half2_rn(act_t<ACT>(v[2 * e], act), act_t<ACT>(v[2 * e + 1], act));
          *reinterpret_cast<uint4 *>(dst + cc) = o;
        }
      }
    }
  }
}

// NT: 128-row tiles per slab, computed together.
template <int BN, int ACT, int NT>
__global__ void __launch_bounds__(kHaloThreads, 1)
    halo_conv_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW,
                     const __grid_constant__ HaloArgs g) {
  constexpr int ACC = acc_cols<BN>();
  constexpr uint32_t TMEM_COLS = 2 * NT * ACC <= 32 ? 32 : 2 * NT * ACC <= 64 ? 64 : 2 * NT * ACC <= 128 ? 128
                                 : 2 * NT * ACC <= 256 ? 256 : 512;
  static_assert(2 * NT * ACC <= 512, "accumulators exceed TMEM");
  constexpr uint32_t TAP_BYTES = BN * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *wsm = smem;                                    // resident filter, 9 taps
  uint8_t *slab0 = smem + ((g.w_bytes + 1023) & ~1023u);  // slab ring
  uint8_t *bars = slab0 + g.nbuf * g.slab_stride + g.slack; // last tile reads past the slab
  uint64_t *full = reinterpret_cast<uint64_t *>(bars);
  uint64_t *empty = full + kMaxBufs;
  uint64_t *tfull = empty + kMaxBufs;
  uint64_t *tempty = tfull + 2;
  uint64_t *wbar = tempty + 2;
  uint64_t *drain = wbar + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile = blockIdx.x % g.ntiles;
  const int first = blockIdx.x / g.ntiles, step = gridDim.x / g.ntiles;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int b = 0; b < kMaxBufs; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(wbar, 1);
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Nothing above touches global memory (programmatic dependent launch).
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&mapX);
      prefetch_tensormap(&mapW);
      mbar_arrive_expect_tx(wbar, g.w_bytes);
      for (int tap = 0; tap < 9; ++tap)
        tma_load_3d(wsm + tap * TAP_BYTES, &mapW, wbar, 0, tap, ntile * BN);
      uint32_t issued = 0, issued_par = 0;
      int it = 0;
      for (int s = first; s < g.slabs; s += step, ++it) {
        const int b = it % g.nbuf;
        const uint32_t par = (it / g.nbuf) & 1;
        if (!mbar_wait(&empty[b], par ^ 1, abort)) {
          halo_fail(g, abort, 11);
          break;
        }
        const int cb = s % g.col_blocks;
        const int rest = s / g.col_blocks;
        const int rb = rest % g.row_blocks;
        const int n = rest / g.row_blocks;
        mbar_arrive_expect_tx(&full[b], g.slab_bytes);
        issued |= 1u << b;
        issued_par = (issued_par & ~(1u << b)) | (par << b);
        // Halo origin: output (rb * R, cb * Wt) minus the padding of 1.
        tma_load_4d(slab0 + b * g.slab_stride, &mapX, &full[b], 0, cb * g.Wt - 1, rb * g.R - 1, n);
      }
      // Every load issued must land before shared memory goes away.
      for (int b = 0; b < kMaxBufs; ++b)
        if (issued & (1u << b)) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[b], (issued_par >> b) & 1u) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
      const long long t0 = clock64();
      while (!mbar_try_wait(wbar, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Every operand address is a fixed offset from two base descriptors
      // (the address field holds addr >> 4 and never carries: shared
      // addresses stay below 256 KB), so each MMA costs one 64-bit add per
      // operand. A 128-byte row is 8 address units, a K step of 16 fp16 is 2.
      const uint32_t idesc = idesc_f16_f32(128, BN);
      const uint64_t bdesc0 = sdesc_k_sw128(smem_u32(wsm));
      const uint32_t wp8 = static_cast<uint32_t>(g.Wp) * 8;
      const int slabs = g.slabs, nbuf = g.nbuf, ks = g.ks;
      const uint32_t slab_stride = g.slab_stride;
      bool ok = mbar_wait(wbar, 0, abort);
      if (!ok)
        halo_fail(g, abort, 12);
      int it = 0;
      for (int s = first; ok && s < slabs; s += step, ++it) {
        const int b = it % nbuf;
        if (!mbar_wait(&full[b], (it / nbuf) & 1, abort)) {
          halo_fail(g, abort, 13);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t adesc0 = sdesc_k_sw128(smem_u32(slab0 + b * slab_stride));
        const int set = it & 1;
        if (!mbar_wait(&tempty[set], ((it >> 1) & 1) ^ 1, abort)) {
          halo_fail(g, abort, 14);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + set * NT * ACC;
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const uint64_t a = adesc0 + (tap / 3) * wp8 + (tap % 3) * 8;
          const uint64_t bt = bdesc0 + tap * (TAP_BYTES >> 4);
          for (int k = 0; k < ks; ++k)
#pragma unroll
            for (int t = 0; t < NT; ++t)
              umma_f16(d + t * ACC, a + t * 128 * 8 + 2 * k, bt + 2 * k, idesc, (tap | k) != 0);
        }
        umma_commit(&tfull[set]);
        if (ok)
          umma_commit(&empty[b]); // the slab is free once its MMAs complete
      }
      umma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else {
    // Epilogue: warp w drains TMEM lane quarter w % 4.
    const int q = warp & 3;
    const int wp = g.Wp, R = g.R, Wt = g.Wt, OH = g.OH, OW = g.OW, ldo = g.ldo, Co = g.Co;
    const int slabs = g.slabs;
    const int n0 = ntile * BN;
    const half *bias = g.bias;
    half *out = g.out;
    bool ok = true;
    int it = 0;
    for (int s = first; ok && s < slabs; s += step, ++it) {
      const int cb = s % g.col_blocks;
      const int rest = s / g.col_blocks;
      const int rb = rest % g.row_blocks;
      const int n = rest / g.row_blocks;
      const int set = it & 1;
      if (!mbar_wait(&tfull[set], (it >> 1) & 1, abort)) {
        halo_fail(g, abort, 15);
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int t = 0; t < NT; ++t)
        halo_drain_tile<BN, ACT>(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + (set * NT + t) * ACC,
                                 t * 128 + q * 32 + lane, wp, R, Wt, rb, cb, n, OH, OW, ldo, n0, Co, bias, out,
                                 g.act);
      tc_fence_before();
      mbar_arrive(&tempty[set]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Streamed-filter form for wide inputs (Ci = 128..1024 in 64-channel chunks)
// and narrow outputs (Co <= 64): the detector's FPN and DB-head 3x3 convs
// (256 -> 64 at 30..240 pixels square).
//
// The generic implicit GEMM loads one 128-byte channel block per pixel per
// tap, nine loads of every input pixel per 64 output channels; with N = 64
// that L2 -> shared-memory traffic (2.7 GB per 240x240x8 layer) is the
// bound. Here a stage is one filter row kh and one 64-channel chunk c: the
// R input rows (oh0 + kh - 1 ..) of the slab as one SW128 TMA box of Wp =
// Wt + 2 pixels per row, plus the three taps (kh, 0..2) of chunk c (3 x 64
// rows of 128 bytes). The kw taps address the box through UMMA descriptors
// shifted by kw rows, exactly as the resident-filter kernel above does for
// all nine taps; the filter cannot stay resident (9 x 256 x 64 fp16 = 295
// KB), so it streams with the activations, once per slab and stage. Per
// slab: 3 x (Ci / 64) stages accumulate into the slab's NT accumulators
// (double-buffered across slabs); input pixels cross L2 -> SM three times
// instead of nine. Roles and bounded waits as in halo_conv_kernel.
struct StreamArgs {
  int OH, OW, batch;
  int R, Wt, Wp;
  int row_blocks, col_blocks, slabs;
  int nck;               // 64-channel input chunks
  int nbuf;              // stage ring depth
  uint32_t a_bytes;      // R * Wp * 128: the TMA box of one stage
  uint32_t a_stride;     // a_bytes + overreach, 1 KB aligned
  uint32_t stage_stride; // a_stride + 3 taps x 64 rows x 128 B
  int Co, ldo;
  const half *bias;
  half *out;
  int act;
  int *err;
};

template <int ACT, int NT>
__global__ void __launch_bounds__(kHaloThreads, 1)
    halo_stream_kernel(const __grid_constant__ CUtensorMap mapX, const __grid_constant__ CUtensorMap mapW,
                       const __grid_constant__ StreamArgs g) {
  constexpr int BN = 64, ACC = 64;
  constexpr uint32_t TMEM_COLS = 2 * NT * ACC <= 128 ? 128 : 2 * NT * ACC <= 256 ? 256 : 512;
  static_assert(2 * NT * ACC <= 512, "accumulators exceed TMEM");
  constexpr uint32_t TAP_BYTES = BN * 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *bars = smem + g.nbuf * g.stage_stride;
  uint64_t *full = reinterpret_cast<uint64_t *>(bars);
  uint64_t *empty = full + kMaxBufs;
  uint64_t *tfull = empty + kMaxBufs;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int first = blockIdx.x, step = gridDim.x;
  const int stages_per_slab = 3 * g.nck;
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int b = 0; b < kMaxBufs; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Nothing above touches global memory (programmatic dependent launch).
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&mapX);
      prefetch_tensormap(&mapW);
      uint32_t issued = 0, issued_par = 0;
      int it = 0;
      bool ok = true;
      for (int s = first; ok && s < g.slabs; s += step) {
        const int cb = s % g.col_blocks;
        const int rest = s / g.col_blocks;
        const int rb = rest % g.row_blocks;
        const int n = rest / g.row_blocks;
        for (int st = 0; st < stages_per_slab; ++st, ++it) {
          const int kh = st / g.nck, c = st - kh * g.nck;
          const int b = it % g.nbuf;
          const uint32_t par = (it / g.nbuf) & 1;
          if (!mbar_wait(&empty[b], par ^ 1, abort)) {
            halo_fail(g.err, abort, 16);
            ok = false;
            break;
          }
          uint8_t *stage = smem + b * g.stage_stride;
          mbar_arrive_expect_tx(&full[b], g.a_bytes + 3 * TAP_BYTES);
          issued |= 1u << b;
          issued_par = (issued_par & ~(1u << b)) | (par << b);
          // Input rows rb * R + kh - 1 .. (+R), columns cb * Wt - 1 .. (+Wp);
          // outside the image the box is zero-filled (the conv padding).
          tma_load_4d(stage, &mapX, &full[b], c * 64, cb * g.Wt - 1, rb * g.R + kh - 1, n);
          for (int kw = 0; kw < 3; ++kw)
            tma_load_3d(stage + g.a_stride + kw * TAP_BYTES, &mapW, &full[b], c * 64, kh * 3 + kw, 0);
        }
      }
      // Every load issued must land before shared memory goes away.
      for (int b = 0; b < kMaxBufs; ++b)
        if (issued & (1u << b)) {
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[b], (issued_par >> b) & 1u) && clock64() - t0 < kWaitBudgetCycles) {
          }
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(128, BN);
      const int slabs = g.slabs, nbuf = g.nbuf;
      bool ok = true;
      int it = 0, sl = 0;
      for (int s = first; ok && s < slabs; s += step, ++sl) {
        const int set = sl & 1;
        if (!mbar_wait(&tempty[set], ((sl >> 1) & 1) ^ 1, abort)) {
          halo_fail(g.err, abort, 17);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + set * NT * ACC;
        for (int st = 0; st < stages_per_slab; ++st, ++it) {
          const int b = it % nbuf;
          if (!mbar_wait(&full[b], (it / nbuf) & 1, abort)) {
            halo_fail(g.err, abort, 18);
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t *stage = smem + b * g.stage_stride;
          const uint64_t a0 = sdesc_k_sw128(smem_u32(stage));
          const uint64_t b0 = sdesc_k_sw128(smem_u32(stage + g.a_stride));
#pragma unroll
          for (int kw = 0; kw < 3; ++kw)
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
              for (int t = 0; t < NT; ++t)
                umma_f16(d + t * ACC, a0 + t * 128 * 8 + kw * 8 + 2 * k, b0 + kw * (TAP_BYTES >> 4) + 2 * k, idesc,
                         (st | kw | k) != 0);
          umma_commit(&empty[b]); // the stage is free once its MMAs complete
        }
        if (ok)
          umma_commit(&tfull[set]);
      }
      umma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else {
    // Epilogue: warp w drains TMEM lane quarter w % 4.
    const int q = warp & 3;
    bool ok = true;
    int sl = 0;
    for (int s = first; ok && s < g.slabs; s += step, ++sl) {
      const int cb = s % g.col_blocks;
      const int rest = s / g.col_blocks;
      const int rb = rest % g.row_blocks;
      const int n = rest / g.row_blocks;
      const int set = sl & 1;
      if (!mbar_wait(&tfull[set], (sl >> 1) & 1, abort)) {
        halo_fail(g.err, abort, 19);
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int t = 0; t < NT; ++t)
        halo_drain_tile<BN, ACT>(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + (set * NT + t) * ACC,
                                 t * 128 + q * 32 + lane, g.Wp, g.R, g.Wt, rb, cb, n, g.OH, g.OW, g.ldo, 0,
                                 g.Co, g.bias, g.out, g.act);
      tc_fence_before();
      mbar_arrive(&tempty[set]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

uint32_t round1k(uint32_t v) { return (v + 1023) & ~1023u; }

size_t halo_smem(uint32_t w_bytes, uint32_t slab_bytes, int nbuf, uint32_t slack) {
  return 1024 + round1k(w_bytes) + nbuf * size_t(round1k(slab_bytes)) + round1k(slack) + 256;
}

// Rows of 128 bytes the last tile of a slab reads past the slab's halo.
uint32_t overreach_bytes(int R, int wp, int tiles) {
  const int rows = tiles * 128 + 2 - R * wp;
  return rows > 0 ? static_cast<uint32_t>(rows) * 128u : 0u;
}

template <int BN, int ACT, int NT>
cudaError_t launch_halo(const CUtensorMap &mx, const CUtensorMap &mw, const HaloArgs &g, size_t smem,
                        cudaStream_t s) {
  auto kernel = halo_conv_kernel<BN, ACT, NT>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit));
  });
  if (attr != cudaSuccess)
    return attr;
  // CTAs come in groups of ntiles (one per N tile) sharing the slab order.
  const long long work = static_cast<long long>(g.slabs) * g.ntiles;
  int grid = sm_count() / g.ntiles * g.ntiles;
  if (work < grid)
    grid = static_cast<int>(work);
  launch_pdl(kernel, grid, kHaloThreads, smem, s, mx, mw, g);
  return cudaGetLastError();
}

template <int BN, int NT>
cudaError_t dispatch_halo_act(const CUtensorMap &mx, const CUtensorMap &mw, const HaloArgs &g, size_t smem,
                              cudaStream_t s) {
  switch (g.act) {
  case kActNone:
    return launch_halo<BN, kActNone, NT>(mx, mw, g, smem, s);
  case kActRelu:
    return launch_halo<BN, kActRelu, NT>(mx, mw, g, smem, s);
  default:
    return launch_halo<BN, -1, NT>(mx, mw, g, smem, s);
  }
}

template <int BN>
cudaError_t dispatch_halo_nt(const CUtensorMap &mx, const CUtensorMap &mw, const HaloArgs &g, size_t smem,
                             cudaStream_t s) {
  switch (g.tiles) {
  case 1:
    return dispatch_halo_act<BN, 1>(mx, mw, g, smem, s);
  case 2:
    return dispatch_halo_act<BN, 2>(mx, mw, g, smem, s);
  case 3:
    return dispatch_halo_act<BN, 3>(mx, mw, g, smem, s);
  default:
    return dispatch_halo_act<BN, 4>(mx, mw, g, smem, s);
  }
}

// Slab shape (R, Wt) and ring depth within the shared-memory budget
// (resident filter + ring + overreach slack): among shapes that waste at
// most 10 % more MMA rows than the best, the one with the most tiles per
// slab (up to 4, interleaved), then the fewest wasted rows.
bool pick_slab(int OH, int OW, uint32_t w_bytes, int &R, int &Wt, int &nbuf) {
  struct Cand {
    int r, wt, nb, tiles;
    double eff;
  };
  Cand cands[16 * 16];
  int nc = 0;
  double best = 0.0;
  for (int cbk = 1; cbk <= 16; ++cbk) {
    const int wt = (OW + cbk - 1) / cbk;
    const int wp = wt + 2;
    if (wp > 256)
      continue;
    for (int r = 1; r <= 16; ++r) {
      const int tiles = (r * wp + 127) / 128;
      if (tiles > 4)
        break;
      const uint32_t slab = static_cast<uint32_t>(r + 2) * wp * 128;
      const uint32_t slack = overreach_bytes(r, wp, tiles);
      int nb = 0;
      for (int k = kMaxBufs; k >= 2 && !nb; --k)
        if (halo_smem(w_bytes, slab, k, slack) <= kSmemLimit)
          nb = k;
      if (!nb)
        break;
      const int rbk = (OH + r - 1) / r;
      const double eff = static_cast<double>(OH) * OW / (static_cast<double>(rbk) * cbk * tiles * 128);
      cands[nc++] = {r, wt, nb, tiles, eff};
      if (eff > best)
        best = eff;
    }
  }
  int pick = -1;
  for (int i = 0; i < nc; ++i) {
    if (cands[i].eff < 0.9 * best)
      continue;
    if (pick < 0 || cands[i].tiles > cands[pick].tiles ||
        (cands[i].tiles == cands[pick].tiles && cands[i].eff > cands[pick].eff + 1e-9))
      pick = i;
  }
  if (pick < 0)
    return false;
  R = cands[pick].r;
  Wt = cands[pick].wt;
  nbuf = cands[pick].nb;
  return true;
}

size_t stream_smem(const StreamArgs &g) { return 1024 + size_t(g.nbuf) * g.stage_stride + 256; }

template <int ACT, int NT>
cudaError_t launch_stream(const CUtensorMap &mx, const CUtensorMap &mw, const StreamArgs &g, cudaStream_t s) {
  auto kernel = halo_stream_kernel<ACT, NT>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit));
  });
  if (attr != cudaSuccess)
    return attr;
  const int grid = g.slabs < sm_count() ? g.slabs : sm_count();
  launch_pdl(kernel, grid, kHaloThreads, stream_smem(g), s, mx, mw, g);
  return cudaGetLastError();
}

template <int NT>
cudaError_t dispatch_stream_act(const CUtensorMap &mx, const CUtensorMap &mw, const StreamArgs &g, cudaStream_t s) {
  switch (g.act) {
  case kActNone:
    return launch_stream<kActNone, NT>(mx, mw, g, s);
  case kActRelu:
    return launch_stream<kActRelu, NT>(mx, mw, g, s);
  default:
    return launch_stream<-1, NT>(mx, mw, g, s);
  }
}

// Slab shape for the streamed form, from a cost model of the persistent
// grid: time ~ waves x tiles per slab x the per-MMA cost of that many
// interleaved accumulators (consecutive MMAs into one accumulator wait on
// each other at N = 64: one tile runs at about half rate, two at 0.8),
// waves = ceil(slabs / SMs). Large layers take 4-tile slabs (the 240^2
// detector layers: 2-row slabs); small ones trade tiles per slab for more
// slabs in flight (30^2 x 8 pages: 64 one-tile slabs instead of 16
// four-tile ones). Ties go to more tiles per slab, then fewer wasted rows.
// The ring is the deepest (2..4 stages) that fits; a stage holds R input
// rows of Wp pixels (+ the overreach of the last tile) and three 8 KB
// filter taps.
bool pick_stream_slab(int batch, int OH, int OW, StreamArgs &g) {
  static const double kTilePenalty[5] = {0.0, 2.0, 1.25, 1.05, 1.0};
  const int sms = sm_count();
  bool found = false;
  double best_cost = 0.0, best_eff = 0.0;
  int best_tiles = 0;
  for (int cbk = 1; cbk <= 16; ++cbk) {
    const int wt = (OW + cbk - 1) / cbk;
    const int wp = wt + 2;
    if (wp > 256)
      continue;
    for (int r = 1; r <= 16 && r <= OH + 15; ++r) {
      const int tiles = (r * wp + 127) / 128;
      if (tiles > 4)
        break;
      const uint32_t a_bytes = static_cast<uint32_t>(r) * wp * 128;
      const uint32_t a_stride = round1k(a_bytes + overreach_bytes(r, wp, tiles));
      const uint32_t stage = a_stride + 3 * 64 * 128;
      int nb = 0;
      for (int k = kMaxBufs; k >= 2 && !nb; --k)
        if (1024 + size_t(k) * stage + 256 <= kSmemLimit)
          nb = k;
      if (!nb)
        break;
      const int rbk = (OH + r - 1) / r;
      const long long slabs = static_cast<long long>(batch) * rbk * cbk;
      const double waves = static_cast<double>((slabs + sms - 1) / sms);
      const double cost = waves * tiles * kTilePenalty[tiles];
      const double eff = static_cast<double>(OH) * OW / (static_cast<double>(rbk) * cbk * tiles * 128);
      const bool better = !found || cost < best_cost * (1 - 1e-9) ||
                          (cost <= best_cost * (1 + 1e-9) &&
                           (tiles > best_tiles || (tiles == best_tiles && eff > best_eff + 1e-9)));
      if (better) {
        found = true;
        best_cost = cost;
        best_eff = eff;
        best_tiles = tiles;
        g.R = r;
        g.Wt = wt;
        g.Wp = wp;
        g.nbuf = nb;
        g.a_bytes = a_bytes;
        g.a_stride = a_stride;
        g.stage_stride = stage;
      }
      if (r >= OH)
        break; // taller slabs only add empty rows
    }
  }
  return found;
}

} // namespace

bool halo_conv_supported(const ConvShape &s, const GemmEpilogue &epi) {
  const int OH = s.out_h ? s.out_h : s.H + 2 * s.pad_h - s.KH + 1;
  const int OW = s.out_w ? s.out_w : s.W + 2 * s.pad_w - s.KW + 1;
  return !epi.residual && s.Ci % 16 == 0 && s.Ci >= 16 && s.Ci <= 64 && s.Co % 16 == 0 && s.Co <= 256 &&
         s.KH == 3 && s.KW == 3 && s.pad_h == 1 && s.pad_w == 1 && OH == s.H && OW == s.W && epi.ldo % 8 == 0;
}

cudaError_t halo_conv(const half *x, const half *w, const ConvShape &s, const GemmEpilogue &epi,
                      cudaStream_t stream) {
  if (!halo_conv_supported(s, epi))
    return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(epi.out) & 15) || (epi.bias && (reinterpret_cast<uintptr_t>(epi.bias) & 15)))
    return cudaErrorInvalidValue;
  // N tile: Co up to 64 in one tile (48 for Co <= 48); wider layers split
  // into 64-column tiles so the resident filter leaves room for the ring.
  const int BN = s.Co <= 48 ? 48 : 64;
  const int ntiles = (s.Co + BN - 1) / BN;
  const uint32_t w_bytes = 9u * BN * 128;
  int R = 0, Wt = 0, nbuf = 0;
  if (!pick_slab(s.H, s.W, w_bytes, R, Wt, nbuf))
    return cudaErrorNotSupported;
  HaloArgs g{};
  g.OH = s.H;
  g.OW = s.W;
  g.batch = s.batch;
  g.R = R;
  g.Wt = Wt;
  g.Wp = Wt + 2;
  g.row_blocks = (s.H + R - 1) / R;
  g.col_blocks = (s.W + Wt - 1) / Wt;
  const long long slabs = static_cast<long long>(s.batch) * g.row_blocks * g.col_blocks;
  if (slabs > 0x3fffffffLL)
    return cudaErrorInvalidValue;
  g.slabs = static_cast<int>(slabs);
  g.ntiles = ntiles;
  g.tiles = (R * g.Wp + 127) / 128;
  g.ks = s.Ci / 16;
  g.nbuf = nbuf;
  g.slab_bytes = static_cast<uint32_t>(R + 2) * g.Wp * 128;
  g.slab_stride = round1k(g.slab_bytes);
  g.w_bytes = w_bytes;
  g.slack = round1k(overreach_bytes(R, g.Wp, g.tiles));
  g.Co = s.Co;
  g.ldo = epi.ldo;
  g.bias = epi.bias;
  g.out = epi.out;
  g.act = epi.act;
  g.err = device_error_word();
  // x [batch][H][W][Ci]: 64-channel boxes of Wp pixels x (R + 2) rows.
  CUtensorMap mx, mw;
  cuuint64_t dx[4] = {static_cast<cuuint64_t>(s.Ci), static_cast<cuuint64_t>(s.W), static_cast<cuuint64_t>(s.H),
                      static_cast<cuuint64_t>(s.batch)};
  cuuint64_t sx[3] = {static_cast<cuuint64_t>(s.Ci) * 2, static_cast<cuuint64_t>(s.W) * s.Ci * 2,
                      static_cast<cuuint64_t>(s.H) * s.W * s.Ci * 2};
  cuuint32_t bx[4] = {64, static_cast<cuuint32_t>(g.Wp), static_cast<cuuint32_t>(R + 2), 1};
  // w [Co][9][Ci]: one 64-channel x BN-row box per tap.
  cuuint64_t dw[3] = {static_cast<cuuint64_t>(s.Ci), 9, static_cast<cuuint64_t>(s.Co)};
  cuuint64_t sw[2] = {static_cast<cuuint64_t>(s.Ci) * 2, static_cast<cuuint64_t>(9) * s.Ci * 2};
  cuuint32_t bw[3] = {64, 1, static_cast<cuuint32_t>(BN)};
  if (!encode_fp16_map(&mx, x, 4, dx, sx, bx, true) || !encode_fp16_map(&mw, w, 3, dw, sw, bw, true))
    return cudaErrorNotSupported;
  const size_t smem = halo_smem(w_bytes, g.slab_bytes, nbuf, g.slack);
  return BN == 48 ? dispatch_halo_nt<48>(mx, mw, g, smem, stream) : dispatch_halo_nt<64>(mx, mw, g, smem, stream);
}

bool halo_stream_supported(const ConvShape &s, const GemmEpilogue &epi) {
  const int OH = s.out_h ? s.out_h : s.H + 2 * s.pad_h - s.KH + 1;
  const int OW = s.out_w ? s.out_w : s.W + 2 * s.pad_w - s.KW + 1;
  return !epi.residual && s.Ci % 64 == 0 && s.Ci >= 128 && s.Ci <= 1024 && s.Co % 16 == 0 && s.Co <= 64 &&
         s.KH == 3 && s.KW == 3 && s.pad_h == 1 && s.pad_w == 1 && OH == s.H && OW == s.W && epi.ldo % 8 == 0;
}

cudaError_t halo_stream_conv(const half *x, const half *w, const ConvShape &s, const GemmEpilogue &epi,
                             cudaStream_t stream) {
  if (!halo_stream_supported(s, epi))
    return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(epi.out) & 15) || (epi.bias && (reinterpret_cast<uintptr_t>(epi.bias) & 15)))
    return cudaErrorInvalidValue;
  if (s.batch <= 0 || s.H <= 0 || s.W <= 0)
    return cudaSuccess;
  StreamArgs g{};
  if (!pick_stream_slab(s.batch, s.H, s.W, g))
    return cudaErrorNotSupported;
  g.OH = s.H;
  g.OW = s.W;
  g.batch = s.batch;
  g.row_blocks = (s.H + g.R - 1) / g.R;
  g.col_blocks = (s.W + g.Wt - 1) / g.Wt;
  const long long slabs = static_cast<long long>(s.batch) * g.row_blocks * g.col_blocks;
  if (slabs > 0x3fffffffLL)
    return cudaErrorInvalidValue;
  g.slabs = static_cast<int>(slabs);
  g.nck = s.Ci / 64;
  g.Co = s.Co;
  g.ldo = epi.ldo;
  g.bias = epi.bias;
  g.out = epi.out;
  g.act = epi.act;
  g.err = device_error_word();
  // x [batch][H][W][Ci]: boxes of 64 channels x Wp pixels x R rows.
  CUtensorMap mx, mw;
  cuuint64_t dx[4] = {static_cast<cuuint64_t>(s.Ci), static_cast<cuuint64_t>(s.W), static_cast<cuuint64_t>(s.H),
                      static_cast<cuuint64_t>(s.batch)};
  cuuint64_t sx[3] = {static_cast<cuuint64_t>(s.Ci) * 2, static_cast<cuuint64_t>(s.W) * s.Ci * 2,
                      static_cast<cuuint64_t>(s.H) * s.W * s.Ci * 2};
  cuuint32_t bx[4] = {64, static_cast<cuuint32_t>(g.Wp), static_cast<cuuint32_t>(g.R), 1};
  // w [Co][9][Ci]: one 64-channel x 64-row box per tap and chunk (rows past
  // Co zero-filled).
  cuuint64_t dw[3] = {static_cast<cuuint64_t>(s.Ci), 9, static_cast<cuuint64_t>(s.Co)};
  cuuint64_t sw[2] = {static_cast<cuuint64_t>(s.Ci) * 2, static_cast<cuuint64_t>(9) * s.Ci * 2};
  cuuint32_t bw[3] = {64, 1, 64};
  if (!encode_fp16_map(&mx, x, 4, dx, sx, bx, true) || !encode_fp16_map(&mw, w, 3, dw, sw, bw, true))
    return cudaErrorNotSupported;
  const int tiles = (g.R * g.Wp + 127) / 128;
  switch (tiles) {
  case 1:
    return dispatch_stream_act<1>(mx, mw, g, stream);
  case 2:
    return dispatch_stream_act<2>(mx, mw, g, stream);
  case 3:
    return dispatch_stream_act<3>(mx, mw, g, stream);
  default:
    return dispatch_stream_act<4>(mx, mw, g, stream);
  }
}

} // namespace pb2
