// tcgen05 tensor-core GEMM and stride-1 implicit-GEMM convolution for sm_100a.
//
// Replaces the reference's 1x1 cublasLt/CUTLASS-Sm80 GEMMs
// (native/src/compiled/runtime.cuh:514-667, cutlass_gemm.cu:20-120), its
// cuDNN dense convolutions (runtime.cuh:766-815) and the WMMA vocabulary
// projection (native/src/kernels/classifier.cu:388-516).
//
// Design: one persistent CTA per SM:
//   warp 0      TMA producer   (one thread) fills a STAGES-deep smem ring
//   warp 1      UMMA issuer    (one thread) tcgen05.mma 128xBNx16 into TMEM
//   warps 2..   epilogue       tcgen05.ld -> fused bias/act/residual -> HBM
//               (4 warps; 16 for the vocabulary argmax/exp reduction)
// The TMEM accumulator is double buffered so the epilogue of tile i overlaps
// the main loop of tile i+1. Operand tiles are K-major, 128-byte swizzled.
//
// Long-K layers use 256-row tiles instead (MH = 2 M halves): both halves
// multiply the same B stage, so a k-block moves 64 KB of operands for
// 2x128x256x64 MACs instead of 48 KB for half of that (a third fewer bytes
// from L2 per FLOP, and 3 x 64 KB of loads in flight). The two halves fill
// all 512 TMEM columns, so the accumulator is single buffered and 8
// epilogue warps (two per lane quarter, one per half) drain it.
//
// Implicit GEMM: output rows are enumerated as (image, out_row, pixel
// segment of 16 or 32); one A stage (128 rows x 64 channels of one filter
// tap) is eight (or four) 4-D TMA boxes of one segment x 64 channels at the
// tap-shifted coordinates.
// TMA zero-fills out-of-range pixels (the convolution padding), channels past
// Ci and images past the batch, so no im2col buffer exists.
#include "kernels.h"
#include "ptx.cuh"
#include <cfloat>
#include <climits>
#include <mutex>
#include <type_traits>
#include <vector>

namespace pb2 {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
// Epilogues: fused store (NHWC / row-major output), vocabulary argmax/exp
// partials, and the transposed-convolution store (each 64-column chunk is
// one filter tap of KH x KW, written to its stride-interleaved output
// pixels through a 5-D tensor map).
// kEpiDbTail: the DB head's last two transposed convs in one pass -- the
// 2x2 stride-2 conv to 64 channels computed on the tensor cores, its fp16
// outputs (bias, activation) reduced on the spot by the following 2x2
// stride-2 conv to one channel (+ bias, sigmoid), so the 64-channel map at
// twice the resolution is never written.
enum Epi : int { kEpiStore = 0, kEpiVocab = 1, kEpiDeconv = 2, kEpiDbTail = 3 };

// Epilogue warps: 8 for stores, two per TMEM lane quarter: with 256-row
// tiles each drains one M half, with 128-row tiles of 128 or 256 columns
// each drains one column half (a lone tile's epilogue is a latency chain per
// warp, so two warps per quarter halve it); 16 for the exp-heavy vocabulary
// reduction (four warps per quarter, 64 columns each) and for the DB tail
// (one 64-column chunk each: 100 us against 125 us with 8 warps at C5).
template <int EPI, int MH> struct EpiWarps {
  static constexpr int value = EPI == kEpiVocab || EPI == kEpiDbTail ? 16 : 8;
};
static_assert(kEpiDeconv != kEpiVocab, "deconv uses the store warps");
template <int EPI, int MH> constexpr int threads_for() {
  return 64 + 32 * EpiWarps<EPI, MH>::value;
}

struct Args {
  int M, N;            // GEMM rows (conv: padded row space), columns
  int num_kb;          // k-blocks per tile
  int kb_per_tap;      // conv: ceil(Ci/64); gemm: num_kb
  int KW, pad_h, pad_w;
  int mt, nt;          // tile grid
  int Wseg, OH, OW, batch; // conv geometry (Wseg = pixel segments per row)
  int seg_log2;            // conv: log2 of the segment length (16 or 32)
  // Long-segment mode (conv, 256-row tiles): an output row is seg_parts
  // segments of seg_len pixels (a multiple of 16, at most 128); a tile is
  // row_segs segments, each loaded as one TMA box per k-block. Tile rows
  // past row_segs * seg_len compute unused values.
  int row_segs;            // 0: pixel-segment mode
  int seg_len, seg_parts;

  GemmEpilogue epi;
  float *part_max;
  int *part_id;
  float *part_sum;
  int part_ld, calc_prob;
  int dec_co, dec_kw; // deconv: output channels, filter width
  // conv mode with a plain 2-D A map: the pixel segments of every tile are
  // consecutive rows of [pixels][Ci] (1x1 over the input pixels with no
  // segment padding), loaded as MH boxes of 128 rows instead of one box per
  // segment (transposed conv; fewer TMA issues for the producer thread)
  int plain_a;
  // kEpiDbTail: the second transposed conv (64 -> 1, 2x2 stride 2): filter
  // as fp32 [64 channels][4 taps], fp16 bias (or null), activation, and its
  // fp16 output [batch][4 H][4 W].
  const float *tail_w;
  const half *tail_bias;
  half *tail_out;
  int tail_act;
  int *err;
};

template <int BN, int MH = 1> struct Cfg {
  static constexpr int BM = kBM * MH;                  // tile rows
  static constexpr uint32_t A_HALF = kBM * kBK * 2;    // one 128-row A block
  static constexpr uint32_t A_BYTES = MH * A_HALF;
  static constexpr uint32_t B_BYTES = BN * kBK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ACC_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  // Accumulator buffers: two (the epilogue of a tile overlaps the main loop
  // of the next) while both fit the 512 TMEM columns, else one.
  static constexpr int NACC = MH * ACC_COLS <= 256 ? 2 : 1;
  static constexpr uint32_t TMEM_COLS = NACC * MH * ACC_COLS;
  // TMA-store epilogue: each of the 8 epilogue warps stages 32 rows x 64
  // columns (4 KB, 128-byte swizzled), then one lane stores it.
  static constexpr bool TMA_EPI = BN % 64 == 0;
  static constexpr uint32_t EPI_BYTES = TMA_EPI ? 8 * 4096 : 0;
  // As many operand stages (up to 8) as the rest of the 227 KB leaves.
  static constexpr int STAGES_FIT = (232448 - 1024 - 256 - EPI_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr size_t SMEM =
      size_t(STAGES) * STAGE_BYTES + EPI_BYTES + 1024 + 256;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N");
  static_assert(MH == 1 || MH == 2, "one or two M halves");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0,
                "TMEM allocation");
  static_assert(B_BYTES % 1024 == 0, "B tile must keep 1024-byte alignment");
  static_assert(SMEM <= 232448, "dynamic shared memory above 227 KB");
};

// Bias and residual of 8 consecutive columns [n0, n0+8) of one output row,
// fetched ahead of the accumulator they are added to, without branches: an
// absent bias or residual (and a row without an output row) reads eight
// fp16 -0, the exact identity of fp16 and fp32 addition (x + -0 = x for
// every x, +0 included); columns at or past N read an in-range column
// instead (their values are never stored).
struct Extra8 {
  uint4 bias, res;
};

__device__ const uint4 kNegZeroHalves = {0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u};

__device__ __forceinline__ Extra8 fetch_extra8(const GemmEpilogue &e, int n0, int N, long long orow) {
  const int nc = n0 + 8 <= N ? n0 : N - 8;
  const uint4 *bp = e.bias ? reinterpret_cast<const uint4 *>(e.bias + nc) : &kNegZeroHalves;
  const uint4 *rp = e.residual && orow >= 0
                        ? reinterpret_cast<const uint4 *>(e.residual + orow * e.ldr + nc)
                        : &kNegZeroHalves;
  return Extra8{__ldg(bp), __ldg(rp)};
}

// Fused epilogue for 8 consecutive columns of one accumulator row:
// v = round(acc) + bias; v = round(v) + residual; y = round(act(v)).
//
// With no activation or ReLU the chain runs in packed fp16 (one conversion,
// then HADD2 / HMAX2 per pair) and gives the same bits as the fp32 formula,
// because rounding the fp32 sum of two fp16 values to fp16 equals rounding
// their exact sum: when their exponents differ by at most 13 the fp32 sum is
// exact, except for a carry out of a 13-apart pair, whose fp32 rounding
// cannot land on an fp16 midpoint; further apart, the smaller operand is
// below an eighth of the larger one's fp16 ulp and both roundings return the
// larger operand (checked exhaustively over all pairs of finite fp16
// values). ReLU commutes with the final rounding. The other activations act
// on the unrounded fp32 sum and keep the fp32 formula.
template <int ACT>
__device__ __forceinline__ uint4 epilogue8(const uint32_t *acc, const GemmEpilogue &e, const Extra8 &x) {
  if constexpr (ACT == kActNone || ACT == kActRelu) {
    uint4 o;
    half2 *h = reinterpret_cast<half2 *>(&o);
    const half2 *bh = reinterpret_cast<const half2 *>(&x.bias);
    const half2 *rh = reinterpret_cast<const half2 *>(&x.res);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // Absent operands are -0 (fetch_extra8): both additions always run.
      h[j] = __float22half2_rn(make_float2(__uint_as_float(acc[2 * j]), __uint_as_float(acc[2 * j + 1])));
      h[j] = __hadd2(__hadd2(h[j], bh[j]), rh[j]);
      if constexpr (ACT == kActRelu)
        h[j] = __hmax2(h[j], __float2half2_rn(0.f));
    }
    return o;
  } else {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = round_half(__uint_as_float(acc[j]));
    {
      const half2 *bh = reinterpret_cast<const half2 *>(&x.bias); // -0 when absent
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(bh[j]);
        v[2 * j] += f.x;
        v[2 * j + 1] += f.y;
      }
    }
    if (e.residual) {
      const half2 *rh = reinterpret_cast<const half2 *>(&x.res);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(rh[j]);
        v[2 * j] = round_half(v[2 * j]) + f.x;
        v[2 * j + 1] = round_half(v[2 * j + 1]) + f.y;
      }
    }
    uint4 o;
    half2 *oh2 = reinterpret_cast<half2 *>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      oh2[j] = __floats2half2_rn(act_t<ACT>(v[2 * j], e.act),
                                 act_t<ACT>(v[2 * j + 1], e.act));
    return o;
  }
}

__device__ __forceinline__ void fail(const Args &g, volatile int *abort,
                                     int code) {
  *abort = 1;
  if (g.err)
    atomicCAS(g.err, 0, code);
}

template <int BN, bool CONV, int EPI, int ACT, int MH>
__global__ void __launch_bounds__(threads_for<EPI, MH>(), 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap mapA,
                   const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapC,
                   const __grid_constant__ Args g) {
  using C = Cfg<BN, MH>;
  constexpr int BM = C::BM;
  constexpr int NACC = C::NACC;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *epi_smem = smem + STAGES * C::STAGE_BYTES; // 1024-aligned
  uint64_t *full = reinterpret_cast<uint64_t *>(epi_smem + C::EPI_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  // [2][4] vocab hand-off (parts 1..3 -> part 0) per (tile parity, lane
  // quarter). One barrier per parity: a part can run one tile ahead of part
  // 0 (the other accumulator), but never two, so a parity wait cannot alias.
  uint64_t *pair = drain + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(pair + 8);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = g.mt * g.nt;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * EpiWarps<EPI, MH>::value);
    }
    mbar_init(drain, 1);
    for (int p = 0; p < 8; ++p)
      mbar_init(&pair[p], 96);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
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
      prefetch_tensormap(&mapA);
      prefetch_tensormap(&mapB);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;     // stages that received at least one load
      uint32_t issued_par = 0; // parity of the last phase armed per stage
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const int mb = tile / g.nt, nb = tile - mb * g.nt;
        // Implicit GEMM: the pixel segments of this M tile (BM/16 of 16
        // pixels or BM/32 of 32) are fixed for the whole K loop; only the
        // filter tap and channel block move.
        const int nbox = g.row_segs ? g.row_segs : BM >> g.seg_log2;
        const int seg0 = mb * nbox;
        // A bytes per stage: whole rows of 128 bytes actually loaded.
        const uint32_t a_bytes = g.row_segs ? static_cast<uint32_t>(g.row_segs * g.seg_len * 128)
                                            : C::A_BYTES;
        // smem row offset (log2 of bytes) between boxes in pixel-segment mode
        const int box_shift = g.seg_log2 + 7;
        int seg_x[BM / 16], seg_y[BM / 16], seg_n[BM / 16];
        if (CONV) {
#pragma unroll
          for (int s = 0; s < BM / 16; ++s) {
            if (g.row_segs) {
              const int sg = seg0 + s; // segment: (n * OH + oh) * parts + part
              const int r = sg / g.seg_parts;
              seg_x[s] = (sg - r * g.seg_parts) * g.seg_len - g.pad_w;
              seg_n[s] = r / g.OH;
              seg_y[s] = r - seg_n[s] * g.OH - g.pad_h;
            } else {
              const int seg = seg0 + s;
              const int r = seg / g.Wseg;
              seg_x[s] = ((seg - r * g.Wseg) << g.seg_log2) - g.pad_w;
              seg_n[s] = r / g.OH;
              seg_y[s] = r - seg_n[s] * g.OH - g.pad_h;
            }
          }
        }
        int cb = 0, tap = 0, kh = 0, kw = 0;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort)) {
            fail(g, abort, 1);
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * C::STAGE_BYTES;
          uint8_t *sb = sa + C::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], a_bytes + C::B_BYTES);
          issued |= 1u << stage;
          issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
          if (CONV) {
            if (g.plain_a) {
#pragma unroll
              for (int h = 0; h < MH; ++h)
                tma_load_2d(sa + h * C::A_HALF, &mapA, &full[stage], cb * kBK, mb * BM + h * kBM);
            } else {
#pragma unroll
              for (int s = 0; s < BM / 16; ++s)
                if (s < nbox)
                  tma_load_4d(sa + (g.row_segs ? s * g.seg_len * 128 : s << box_shift), &mapA,
                              &full[stage], cb * kBK, seg_x[s] + kw, seg_y[s] + kh, seg_n[s]);
            }
            tma_load_3d(sb, &mapB, &full[stage], cb * kBK, tap, nb * BN);
            if (++cb == g.kb_per_tap) {
              cb = 0;
              ++tap;
              if (++kw == g.KW) {
                kw = 0;
                ++kh;
              }
            }
          } else {
#pragma unroll
            for (int h = 0; h < MH; ++h)
              tma_load_2d(sa + h * C::A_HALF, &mapA, &full[stage], kb * kBK,
                          mb * BM + h * kBM);
            tma_load_2d(sb, &mapB, &full[stage], kb * kBK, nb * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Let every load we issued land before the CTA's smem goes away.
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) {
            const uint32_t par = (issued_par >> s) & 1u;
            long long t0 = clock64();
            while (!mbar_try_wait(&full[s], par) &&
                   clock64() - t0 < kWaitBudgetCycles) {
            }
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const int acc = it % NACC;
        const uint32_t acc_phase = (it / NACC) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort)) {
          fail(g, abort, 2);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * MH * C::ACC_COLS;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort)) {
            fail(g, abort, 3);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b0 = a0 + C::A_BYTES;
#pragma unroll
          for (int h = 0; h < MH; ++h)
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              umma_f16(d + h * C::ACC_COLS, sdesc_k_sw128(a0 + h * C::A_HALF + k * 32),
                       sdesc_k_sw128(b0 + k * 32), idesc, (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok)
          umma_commit(&tfull[acc]);
      }
      // Make sure no UMMA is still writing TMEM when it is released.
      umma_commit(drain);
      long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  } else {
    // Epilogue warps: TMEM lane quarter is fixed by warp id modulo 4.
    const int q = warp & 3;          // TMEM lane quarter
    const int hf = (warp - 2) >> 2;  // vocab: column quarter; stores: M or column half
    // M half drained by this warp (DB tail: 16 warps, 4 per lane quarter,
    // each one 64-column tap chunk of one M half)
    const int mh = MH == 2 ? (EPI == kEpiDbTail ? (hf & 1) : hf) : 0;
    const int row_in_tile = mh * kBM + q * 32 + lane;
    const int ew = warp - 2;         // epilogue warp index (staging buffer)
    // Stores with 128-row tiles of 128 or 256 columns: the two warps of a
    // lane quarter drain one column half each. Narrower 128-row tiles are
    // drained by the first four warps; the other four only release the
    // accumulator.
    constexpr bool kColSplit = EPI != kEpiVocab && MH == 1 && BN >= 128;
    const bool drains = EPI == kEpiVocab || MH == 2 || kColSplit || hf == 0;
    const int c_lo = kColSplit ? hf * (BN / 2) : 0;
    const int c_hi = kColSplit ? c_lo + BN / 2 : BN;
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const int mb = tile / g.nt, nb = tile - mb * g.nt;
      const int acc = it % NACC;
      const uint32_t acc_phase = (it / NACC) & 1;
      // Map this thread's accumulator row to an output row.
      long long orow = -1;
      if (CONV && g.row_segs) {
        const int sidx = row_in_tile / g.seg_len;
        const int sg = mb * g.row_segs + sidx;
        const int r = sg / g.seg_parts;
        const int n = r / g.OH;
        if (sidx < g.row_segs && n < g.batch)
          orow = static_cast<long long>(r) * g.OW + (sg - r * g.seg_parts) * g.seg_len +
                 (row_in_tile - sidx * g.seg_len);
      } else if (CONV) {
        const int seg = mb * (BM >> g.seg_log2) + (row_in_tile >> g.seg_log2);
        const int r = seg / g.Wseg;
        const int owseg = seg - r * g.Wseg;
        const int n = r / g.OH;
        const int oh = r - n * g.OH;
        const int ow = (owseg << g.seg_log2) +
                       (row_in_tile & ((1 << g.seg_log2) - 1));
        if (n < g.batch && ow < g.OW)
          orow = (static_cast<long long>(n) * g.OH + oh) * g.OW + ow;
      } else {
        const int m = mb * BM + row_in_tile;
        if (m < g.M)
          orow = m;
      }
      // Residual row of this output row (the row itself, or its nearest 2x
      // source pixel for an upsampled residual).
      long long rrow = orow;
      if (!CONV && g.epi.res_up && orow >= 0) {
        const long long ow2 = 2LL * g.epi.res_w, img = 2LL * g.epi.res_h * ow2;
        const long long n = orow / img, rem = orow - n * img, y = rem / ow2, x = rem - y * ow2;
        rrow = (n * g.epi.res_h + (y >> 1)) * g.epi.res_w + (x >> 1);
      }
      const int n_base = nb * BN;
      // Bias and residual of this warp's first 64-column chunk are fetched
      // before the accumulator wait, each later chunk's while the previous
      // one is stored: their load latency overlaps the tile's main loop and
      // the stores instead of sitting in the epilogue's critical path.
      Extra8 nx[8];
      if constexpr ((EPI == kEpiStore || EPI == kEpiDeconv) && C::TMA_EPI) {
        if (drains) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            nx[j] = fetch_extra8(g.epi, n_base + c_lo + 8 * j, g.N, rrow);
        }
      }
      if (!mbar_wait(&tfull[acc], acc_phase, abort)) {
        fail(g, abort, 4);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             (acc * MH + mh) * C::ACC_COLS;
      if constexpr ((EPI == kEpiStore || EPI == kEpiDeconv) && C::TMA_EPI) {
        // 64-column chunks: TMEM -> registers -> fused epilogue -> swizzled
        // smem row (this thread's row) -> one TMA store per warp. TMA drops
        // rows past M / past the image width and columns past N.
        const GemmEpilogue &e = g.epi;
        // TMA store coordinates of this warp's 32 rows, fixed for the tile
        // (the column coordinate moves per chunk): one piece for plain
        // GEMMs, two 16-row pieces of long segments (seg_len is a multiple
        // of 16, so a piece lies inside one segment), or 32 >> seg_log2
        // pixel segments; piece h is staged at h << piece_shift.
        int npieces = 1, piece_shift = 0;
        int sx[2] = {0, 0}, sy[2] = {0, 0}, sz[2] = {0, 0};
        bool sok[2] = {true, false};
        if (CONV && g.row_segs) {
          npieces = 2;
          piece_shift = 11;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row0 = mh * kBM + q * 32 + h * 16;
            const int sidx = row0 / g.seg_len;
            const int sg = mb * g.row_segs + sidx;
            const int rr = sg / g.seg_parts;
            const int n = rr / g.OH;
            sok[h] = sidx < g.row_segs && n < g.batch;
            sx[h] = (sg - rr * g.seg_parts) * g.seg_len + row0 - sidx * g.seg_len;
            sy[h] = rr - n * g.OH;
            sz[h] = n;
          }
        } else if (CONV) {
          npieces = 32 >> g.seg_log2;
          piece_shift = g.seg_log2 + 7;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int seg = mb * (BM >> g.seg_log2) + ((mh * kBM + q * 32) >> g.seg_log2) + h;
            const int rr = seg / g.Wseg;
            sok[h] = h < npieces;
            sx[h] = (seg - rr * g.Wseg) << g.seg_log2;
            if constexpr (EPI == kEpiDeconv) {
              sy[h] = rr; // the input row n * H + h
            } else {
              const int n = rr / g.OH;
              sy[h] = rr - n * g.OH;
              sz[h] = n;
            }
          }
        } else {
          sx[0] = mb * BM + mh * kBM + q * 32;
        }
#pragma unroll 1
        for (int c = drains ? c_lo : c_hi; c < c_hi; c += 64) {
          uint32_t r[64];
          tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(r));
          tmem_ld16(taddr + c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
          tmem_ld16(taddr + c + 32, *reinterpret_cast<uint32_t(*)[16]>(r + 32));
          tmem_ld16(taddr + c + 48, *reinterpret_cast<uint32_t(*)[16]>(r + 48));
          tmem_ld_wait();
          uint4 packed[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            packed[j] = epilogue8<ACT>(r + 8 * j, e, nx[j]);
          if (c + 64 < c_hi) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              nx[j] = fetch_extra8(e, n_base + c + 64 + 8 * j, g.N, rrow);
          }
          // The store issued from this warp's buffer for the previous chunk
          // must have read its source before the buffer is overwritten.
          if (lane == 0)
            bulk_wait_read<0>();
          __syncwarp();
          uint8_t *buf = epi_smem + ew * 4096;
          uint8_t *row = buf + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4 *>(row + ((j ^ (lane & 7)) << 4)) =
                packed[j];
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI == kEpiDeconv) {
              // Columns [n_base + c, +64) are channels co0.. of tap (a, b).
              const int tap = (n_base + c) / g.dec_co;
              const int co0 = n_base + c - tap * g.dec_co;
              const int a = tap / g.dec_kw;
#pragma unroll
              for (int h = 0; h < 2; ++h)
                if (h < npieces)
                  tma_store_5d(&mapC, buf + (h << piece_shift), co0, tap - a * g.dec_kw, sx[h], a, sy[h]);
            } else if (CONV) {
#pragma unroll
              for (int h = 0; h < 2; ++h)
                if (h < npieces && sok[h])
                  tma_store_4d(&mapC, buf + (h << piece_shift), n_base + c, sx[h], sy[h], sz[h]);
            } else {
              tma_store_2d(&mapC, buf, n_base + c, sx[0]);
            }
            bulk_commit();
          }
        }
      } else if constexpr (EPI == kEpiStore) {
        const GemmEpilogue &e = g.epi;
#pragma unroll 1
        for (int c = drains ? 0 : BN; c < BN; c += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + c, r);
          tmem_ld_wait();
          if (orow >= 0) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int n0 = n_base + c + h * 8;
              if (n0 + 8 > g.N)
                continue;
              *reinterpret_cast<uint4 *>(e.out + orow * e.ldo + n0) =
                  epilogue8<ACT>(r + 8 * h, e, fetch_extra8(e, n0, g.N, rrow));
            }
          }
        }
      } else if constexpr (EPI == kEpiDbTail) {
        // This thread's row is input pixel (n, ih, iw); each 64-column chunk
        // is tap (a, b) of the first transposed conv, i.e. the 64 channels
        // of pixel (2 ih + a, 2 iw + b) at twice the resolution, exactly as
        // the unfused layer would store them (epilogue8: fp16 rounding,
        // bias, activation). The second conv maps that pixel to the 2 x 2
        // block (2 (2 ih + a) + ki, 2 (2 iw + b) + kj) of the output with
        // the arithmetic of its standalone kernel (deconv_group_kernel in
        // detect.cu, eight lanes of eight channels): per group of eight
        // channels one fp32 FMA chain in channel order, the eight group
        // sums added as ((g0+g4) + (g2+g6)) + ((g1+g5) + (g3+g7)), then
        // round to fp16, + bias, activation, fp16 store -- bit-identical.
        const GemmEpilogue &e = g.epi;
        // Tile rows are the input pixels in order (a plain [B*H*W][Ci]
        // operand: two TMA boxes per k-block instead of one per segment).
        const int m = mb * BM + row_in_tile;
        const bool valid = m < g.M;
        const int hw = g.OH * g.OW;
        const int n = m / hw, ih = (m - n * hw) / g.OW, iw = m - n * hw - ih * g.OW;
        const long long OW2 = 4LL * g.OW;
        const float tb = g.tail_bias ? __half2float(*g.tail_bias) : 0.f;
        // The (M half, 64-column chunk) pairs of the tile are dealt to the
        // warps of each TMEM lane quarter in turn; a warp's pairs share its
        // M half. A chunk is one tap of the first conv.
        constexpr int kWq = EpiWarps<EPI, MH>::value / 4;
        // Per warp, in its 2 KB of the (otherwise unused) store-staging
        // smem, once: the second filter, fp32 [64 channels][4 taps], read as
        // broadcast 16-byte loads, and the first conv's bias for all N = 256
        // columns (fp16 -0 when absent, as fetch_extra8 gives).
        float *wsm = reinterpret_cast<float *>(epi_smem + ew * 2048);
        uint4 *bsm = reinterpret_cast<uint4 *>(epi_smem + ew * 2048 + 1024);
        if (it == 0) {
          for (int i = lane; i < 256; i += 32)
            wsm[i] = g.tail_w[i];
          bsm[lane] = e.bias ? *reinterpret_cast<const uint4 *>(e.bias + 8 * lane)
                             : make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
          __syncwarp();
        }
#pragma unroll 1
        for (int pr = hf; pr < MH * (BN / 64); pr += kWq) {
          const int c = pr / MH * 64;
          const uint4 *bchunk = bsm + (n_base + c) / 8;
          float ps[4][8]; // group sums per output tap
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t r[32];
            tmem_ld16(taddr + c + 32 * half, *reinterpret_cast<uint32_t(*)[16]>(r));
            tmem_ld16(taddr + c + 32 * half + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int gi = half * 4 + k;
              Extra8 x;
              x.bias = bchunk[gi];
              x.res = make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
              const uint4 hv = epilogue8<ACT>(r + 8 * k, e, x);
              const half2 *h2 = reinterpret_cast<const half2 *>(&hv);
              float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(h2[j]);
                const float4 w0 = *reinterpret_cast<const float4 *>(wsm + (gi * 8 + 2 * j) * 4);
                const float4 w1 = *reinterpret_cast<const float4 *>(wsm + (gi * 8 + 2 * j + 1) * 4);
                a0 = fmaf(f.x, w0.x, a0);
                a1 = fmaf(f.x, w0.y, a1);
                a2 = fmaf(f.x, w0.z, a2);
                a3 = fmaf(f.x, w0.w, a3);
                a0 = fmaf(f.y, w1.x, a0);
                a1 = fmaf(f.y, w1.y, a1);
                a2 = fmaf(f.y, w1.z, a2);
                a3 = fmaf(f.y, w1.w, a3);
              }
              ps[0][gi] = a0;
              ps[1][gi] = a1;
              ps[2][gi] = a2;
              ps[3][gi] = a3;
            }
          }
          if (valid) {
            float sum[4];
#pragma unroll
            for (int o = 0; o < 4; ++o)
              sum[o] = ((ps[o][0] + ps[o][4]) + (ps[o][2] + ps[o][6])) + ((ps[o][1] + ps[o][5]) + (ps[o][3] + ps[o][7]));
            const int tap = (n_base + c) / g.dec_co;
            const int a = tap / g.dec_kw, b = tap - a * g.dec_kw;
#pragma unroll
            for (int ki = 0; ki < 2; ++ki) {
              float v0 = round_half(sum[2 * ki]), v1 = round_half(sum[2 * ki + 1]);
              if (g.tail_bias) {
                v0 += tb;
                v1 += tb;
              }
              const long long row = 4LL * ih + 2 * a + ki;
              *reinterpret_cast<half2 *>(g.tail_out + (static_cast<long long>(n) * 4 * g.OH + row) * OW2 +
                                         4LL * iw + 2 * b) =
                  __floats2half2_rn(apply_act(v0, g.tail_act), apply_act(v1, g.tail_act));
            }
          }
        }
      } else if constexpr (EPI == kEpiVocab) {
        // Vocabulary tile: fp32 logits = acc + bias, reduced to
        // (max, lowest argmax, sum exp(l - max)) without leaving registers.
        // Four warps share each TMEM lane quarter, each reducing 64 of the
        // tile's 256 columns: the 64 accumulators are read from TMEM once
        // (four loads, one wait, the bias loads in between), then a max pass
        // and an exp pass run on registers with 4 independent accumulator
        // lanes (breaks the compare/add dependency chains). Parts 1..3 hand
        // their result to part 0 through shared memory (double-buffered by
        // tile parity) and the per-parity hand-off mbarrier; part 0 merges
        // in column order and writes the tile's partial.
        constexpr int PART = BN / 4;
        static_assert(PART == 64, "vocabulary parts are 64 columns");
        const int n_lo = n_base + hf * PART;
        const int valid = min(PART, g.N - n_lo); // columns of this part < N
        uint32_t r[PART];
        tmem_ld16(taddr + hf * PART, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(taddr + hf * PART + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld16(taddr + hf * PART + 32, *reinterpret_cast<uint32_t(*)[16]>(r + 32));
        tmem_ld16(taddr + hf * PART + 48, *reinterpret_cast<uint32_t(*)[16]>(r + 48));
        const bool vec_bias =
            valid == PART && (reinterpret_cast<uintptr_t>(g.epi.bias) & 15) == 0;
        tmem_ld_wait();
        // Logits = accumulators + bias (L1-resident, 16-byte loads), 8
        // columns at a time.
        float lg[PART];
        if (vec_bias) {
#pragma unroll
          for (int j8 = 0; j8 < PART / 8; ++j8) {
            const uint4 bb = __ldg(reinterpret_cast<const uint4 *>(g.epi.bias + n_lo + 8 * j8));
            const uint32_t bw[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float lo = __uint_as_float(r[8 * j8 + 2 * j]);
              float hi = __uint_as_float(r[8 * j8 + 2 * j + 1]);
              add2_h(lo, hi, bw[j]); // + fp16 bias, one instruction each
              lg[8 * j8 + 2 * j] = lo;
              lg[8 * j8 + 2 * j + 1] = hi;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < PART; ++j)
            lg[j] = j < valid ? __uint_as_float(r[j]) + __half2float(g.epi.bias[n_lo + j])
                              : -FLT_MAX;
        }
        float bm[4] = {-FLT_MAX, -FLT_MAX, -FLT_MAX, -FLT_MAX};
        int bi[4] = {INT_MAX, INT_MAX, INT_MAX, INT_MAX};
        // Whole parts (all but the vocabulary's last tile) skip the
        // per-column range test.
        auto max_pass = [&](auto whole) {
#pragma unroll
          for (int j = 0; j < PART; ++j)
            if ((decltype(whole)::value || j < valid) && lg[j] > bm[j & 3]) {
              bm[j & 3] = lg[j];
              bi[j & 3] = n_lo + j;
            }
        };
        if (valid == PART)
          max_pass(std::true_type{});
        else
          max_pass(std::false_type{});
        float best = bm[0];
        int best_id = bi[0];
#pragma unroll
        for (int k = 1; k < 4; ++k)
          if (bm[k] > best || (bm[k] == best && bi[k] < best_id)) {
            best = bm[k];
            best_id = bi[k];
          }
        float sum = 0.f;
        if (g.calc_prob && valid > 0) {
          // exp(l - best) = 2^(l*log2e - best*log2e)
          const float bL = best * kLog2e;
          float sp[4] = {0.f, 0.f, 0.f, 0.f};
          auto exp_pass = [&](auto whole) {
#pragma unroll
            for (int j = 0; j < PART; ++j)
              if (decltype(whole)::value || j < valid)
                sp[j & 3] += ex2_ftz(fmaf(lg[j], kLog2e, -bL));
          };
          if (valid == PART)
            exp_pass(std::true_type{});
          else
            exp_pass(std::false_type{});
          sum = (sp[0] + sp[1]) + (sp[2] + sp[3]);
        }
        // Hand-off buffer: [parity][quarter][part 1..3][max | id | sum][lane].
        float *xb = reinterpret_cast<float *>(epi_smem) + ((it & 1) * 4 + q) * 3 * 96;
        if (hf > 0) {
          float *mine = xb + (hf - 1) * 96;
          mine[lane] = best;
          reinterpret_cast<int *>(mine)[32 + lane] = best_id;
          mine[64 + lane] = sum;
          mbar_arrive(&pair[(it & 1) * 4 + q]);
        } else {
          if (!mbar_wait(&pair[(it & 1) * 4 + q], (it >> 1) & 1, abort)) {
            fail(g, abort, 5);
            break;
          }
          float m = best;
          int id = best_id;
          float ms[4], ss[4];
          ms[0] = best;
          ss[0] = sum;
#pragma unroll
          for (int p = 1; p < 4; ++p) {
            const float *theirs = xb + (p - 1) * 96;
            ms[p] = theirs[lane];
            ss[p] = theirs[64 + lane];
            const int pid = reinterpret_cast<const int *>(theirs)[32 + lane];
            if (ms[p] > m) { // parts are in column order: ties keep the lower id
              m = ms[p];
              id = pid;
            }
          }
          float total_sum = 0.f;
#pragma unroll
          for (int p = 0; p < 4; ++p)
            total_sum += ss[p] == 0.f ? 0.f : ss[p] * __expf(ms[p] - m);
          if (orow >= 0) {
            const long long pidx = static_cast<long long>(nb) * g.part_ld + orow;
            g.part_max[pidx] = m;
            g.part_id[pidx] = id;
            g.part_sum[pidx] = total_sum;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
    // Output tiles must be fully written before the CTA exits.
    if (C::TMA_EPI && lane == 0)
      bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ----------------------------------------------------------- host helpers
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                 void *, const cuuint64_t *, const cuuint64_t *,
                                 const cuuint32_t *, const cuuint32_t *,
                                 CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault,
                                &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// fp16 tensor map, innermost dimension first; strides in bytes for dims 1..
bool encode(CUtensorMap *m, const void *base, int rank, const cuuint64_t *dims,
            const cuuint64_t *strides, const cuuint32_t *box) {
  EncodeTiled fn = encoder();
  if (!fn)
    return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank,
                  const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, bool CONV, int EPI, int ACT, int MH = 1>
cudaError_t launch(const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &c,
                   const Args &g,
                   cudaStream_t stream) {
  using C = Cfg<BN, MH>;
  auto kernel = tc_gemm_kernel<BN, CONV, EPI, ACT, MH>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr = cudaSuccess;
  std::call_once(once[dev & 63], [&] {
    attr = cudaFuncSetAttribute(kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(C::SMEM));
  });
  if (attr != cudaSuccess)
    return attr;
  const int total = g.mt * g.nt;
  const int grid = total < sm_count() ? total : sm_count();
  return launch_pdl(kernel, grid, threads_for<EPI, MH>(), C::SMEM, stream, a, b, c, g);
}

// Picks the UMMA N tile that pads the column count least (ties: larger).
int pick_bn(int N) {
  const int cands[] = {256, 128, 64, 48};
  int best = 256;
  long long best_pad = -1;
  for (int bn : cands) {
    if (bn == 48 && N > 48)
      continue;
    long long padded = (static_cast<long long>(N) + bn - 1) / bn * bn;
    if (best_pad < 0 || padded < best_pad) {
      best_pad = padded;
      best = bn;
    }
  }
  return best;
}

// Activations used by the generated graphs get their own instantiation; the
// rest share one with a runtime switch.
template <int BN, bool CONV, int EPI, int MH = 1>
cudaError_t dispatch_act(const CUtensorMap &a, const CUtensorMap &b,
                         const CUtensorMap &c, const Args &g, cudaStream_t s) {
  switch (g.epi.act) {
  case kActNone:
    return launch<BN, CONV, EPI, kActNone, MH>(a, b, c, g, s);
  case kActRelu:
    return launch<BN, CONV, EPI, kActRelu, MH>(a, b, c, g, s);
  case kActHardSwish:
    return launch<BN, CONV, EPI, kActHardSwish, MH>(a, b, c, g, s);
  case kActSwish:
    return launch<BN, CONV, EPI, kActSwish, MH>(a, b, c, g, s);
  default:
    return launch<BN, CONV, EPI, -1, MH>(a, b, c, g, s);
  }
}

// 256-row tiles pay off when the K loop is long (the single-buffered
// accumulator leaves the epilogue exposed once per tile) and there are
// still at least four 256-row tiles per SM (wave quantisation).
bool use_two_halves(int bn, int num_kb, long long M, int nt) {
  return bn == 256 && num_kb >= 32 &&
         (M + 2 * kBM - 1) / (2 * kBM) * nt >= 4LL * sm_count();
}

// 256-row tiles exist for N tiles of 64, 128 and 256.
template <bool CONV, int EPI>
cudaError_t dispatch_bn(int bn, bool two_halves, const CUtensorMap &a,
                        const CUtensorMap &b, const CUtensorMap &c,
                        const Args &g, cudaStream_t s) {
  if constexpr (CONV) {
    if (two_halves && bn != 48) {
      switch (bn) {
      case 64:
        return dispatch_act<64, CONV, EPI, 2>(a, b, c, g, s);
      case 128:
        return dispatch_act<128, CONV, EPI, 2>(a, b, c, g, s);
      default:
        return dispatch_act<256, CONV, EPI, 2>(a, b, c, g, s);
      }
    }
  } else {
    if (two_halves) {
      switch (bn) {
      case 64:
        return dispatch_act<64, CONV, EPI, 2>(a, b, c, g, s);
      case 128:
        return dispatch_act<128, CONV, EPI, 2>(a, b, c, g, s);
      case 256:
        return dispatch_act<256, CONV, EPI, 2>(a, b, c, g, s);
      default:
        break;
      }
    }
  }
  switch (bn) {
  case 48:
    return dispatch_act<48, CONV, EPI>(a, b, c, g, s);
  case 64:
    return dispatch_act<64, CONV, EPI>(a, b, c, g, s);
  case 128:
    return dispatch_act<128, CONV, EPI>(a, b, c, g, s);
  default:
    return dispatch_act<256, CONV, EPI>(a, b, c, g, s);
  }
}

bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

} // namespace

int vocab_tiles(int V) { return (V + 255) / 256; }

bool encode_fp16_map(CUtensorMap *m, const void *base, int rank,
                     const cuuint64_t *dims, const cuuint64_t *strides,
                     const cuuint32_t *box, bool swizzle128) {
  EncodeTiled fn = encoder();
  if (!fn)
    return false;
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void *>(base),
            dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t tc_gemm(const half *A, int M, int K, int lda, const half *W, int N,
                    int ldw, const GemmEpilogue &epi, cudaStream_t stream) {
  if (M <= 0 || N <= 0)
    return cudaSuccess;
  if (K <= 0 || N % 8 || lda % 8 || ldw % 8 || epi.ldo % 8 || !aligned16(A) ||
      !aligned16(W) || !aligned16(epi.out) ||
      (epi.bias && !aligned16(epi.bias)) ||
      (epi.residual && (!aligned16(epi.residual) || epi.ldr % 8)))
    return cudaErrorInvalidValue;
  if (epi.res_up && (!epi.residual || epi.res_h <= 0 || epi.res_w <= 0 ||
                     static_cast<long long>(M) % (4LL * epi.res_h * epi.res_w) != 0))
    return cudaErrorInvalidValue;
  int bn = pick_bn(N);
  const int num_kb = (K + kBK - 1) / kBK;
  // 256-row tiles: long K at N = 256 (see use_two_halves), or a short K
  // loop at N <= 128, where the epilogue dominates and 8 epilogue warps with
  // a double-buffered accumulator drain twice the rows per tile. Very short K
  // (<= 8 k-blocks) at N >= 256 takes 256 x 128 tiles for the same reason
  // (measured: 1x1 512 -> 512 over 245,760 rows 0.141 -> 0.129 ms; at 16
  // k-blocks the extra A re-reads cost more than the epilogue gains).
  bool two = use_two_halves(bn, num_kb, M, (N + bn - 1) / bn) ||
             ((bn == 64 || bn == 128) && num_kb <= 4 &&
              (M + 2 * kBM - 1) / (2 * kBM) * ((N + bn - 1) / bn) >= 2LL * sm_count());
  if (!two && bn == 256 && num_kb <= 8 && N % 128 == 0 &&
      (M + 2 * kBM - 1) / (2 * kBM) * (N / 128) >= 2LL * sm_count()) {
    bn = 128;
    two = true;
  }
  CUtensorMap ma, mb;
  cuuint64_t da[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  cuuint64_t sa[1] = {static_cast<cuuint64_t>(lda) * 2};
  cuuint32_t ba[2] = {kBK, kBM};
  cuuint64_t db[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t sb[1] = {static_cast<cuuint64_t>(ldw) * 2};
  cuuint32_t bb[2] = {kBK, static_cast<cuuint32_t>(bn)};
  // Output map for the TMA-store epilogue: box of 64 columns x 32 rows.
  CUtensorMap mc;
  cuuint64_t dc[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
  cuuint64_t sc[1] = {static_cast<cuuint64_t>(epi.ldo) * 2};
  cuuint32_t bc[2] = {64, 32};
  if (!encode(&ma, A, 2, da, sa, ba) || !encode(&mb, W, 2, db, sb, bb) ||
      !encode(&mc, epi.out, 2, dc, sc, bc))
    return cudaErrorInvalidValue;
  Args g{};
  g.M = M;
  g.N = N;
  g.num_kb = num_kb;
  g.kb_per_tap = g.num_kb;
  g.KW = 1;
  const int bm = two ? 2 * kBM : kBM;
  g.mt = (M + bm - 1) / bm;
  g.nt = (N + bn - 1) / bn;
  g.Wseg = g.OH = g.OW = g.batch = 1;
  g.seg_log2 = 4;
  g.epi = epi;
  g.err = device_error_word();
  return dispatch_bn<false, kEpiStore>(bn, two, ma, mb, mc, g, stream);
}

cudaError_t tc_conv(const half *x, const half *w, const ConvShape &s,
                    const GemmEpilogue &epi, cudaStream_t stream) {
  const int OH = s.out_h ? s.out_h : s.H + 2 * s.pad_h - s.KH + 1;
  const int OW = s.out_w ? s.out_w : s.W + 2 * s.pad_w - s.KW + 1;
  if (s.batch <= 0 || OH <= 0 || OW <= 0)
    return cudaSuccess;
  if (OH > s.H + 2 * s.pad_h - s.KH + 1 || OW > s.W + 2 * s.pad_w - s.KW + 1)
    return cudaErrorInvalidValue;
  if (s.Ci % 8 || s.Co % 8 || epi.ldo % 8 || !aligned16(x) || !aligned16(w) ||
      !aligned16(epi.out) || (epi.bias && !aligned16(epi.bias)) ||
      (epi.residual && (!aligned16(epi.residual) || epi.ldr % 8)) ||
      s.KH * s.KW > 256)
    return cudaErrorInvalidValue;
  if (halo_conv_supported(s, epi)) {
    const cudaError_t e = halo_conv(x, w, s, epi, stream);
    if (e != cudaErrorNotSupported)
      return e;
  }
  if (halo_stream_supported(s, epi)) {
    const cudaError_t e = halo_stream_conv(x, w, s, epi, stream);
    if (e != cudaErrorNotSupported)
      return e;
  }
  int bn = pick_bn(s.Co);
  const int taps = s.KH * s.KW;
  // Segment length: 32 pixels when that pads the output row no more than
  // 16-pixel segments do (half the TMA boxes per stage: OW = 30, 60, 120 of
  // the detector, multiples of 32), else 16. Pixels past OW are zero-filled
  // on load and not stored.
  const int pad16 = (OW + 15) / 16 * 16, pad32 = (OW + 31) / 32 * 32;
  const int seg_log2 = pad32 <= pad16 ? 5 : 4;
  const cuuint32_t seg = 1u << seg_log2;
  const int kb_tap = (s.Ci + kBK - 1) / kBK;
  const int num_kb = kb_tap * taps;
  // Long-segment mode: 256-row tiles of whole output rows, or of equal
  // parts of a row, one TMA box per part and k-block. The part length is
  // the longest divisor of OW that is a multiple of 16, at most 128 and
  // leaves at most one eighth of the tile unused.
  int seg_len = 0;
  for (int parts = 1; parts * 16 <= OW && !seg_len; ++parts) {
    const int len = OW / parts;
    if (OW % parts || len % 16 || len > kBM)
      continue;
    if ((2 * kBM / len) * len * 8 >= 7 * 2 * kBM)
      seg_len = len;
  }
  // Co = 48 with whole-row segments runs as 64-wide tiles of 256 rows: the
  // extra 16 columns cost idle MMA cycles, but a 256-row tile needs 3-4 TMA
  // boxes per k-block where 128-row tiles of 16-pixel segments need 9 (the
  // single producer thread was the limit); columns past Co are neither
  // loaded (zero-filled weights) nor stored.
  if (bn == 48 && seg_len)
    bn = 64;
  int row_segs = 0;
  bool two = false;
  // Measured on B200: 256x256 tiles for long K at N >= 256; 256x128 and
  // 256x64 tiles for N of 128 / 64 (and 48, above); short-K N >= 256 layers
  // and widths without a long segment keep 128-row tiles of 16/32-pixel
  // segments.
  if (seg_len && ((bn == 256 && num_kb >= 16) || bn == 128 || bn == 64)) {
    const long long segs = static_cast<long long>(s.batch) * OH * (OW / seg_len);
    const int per_tile = 2 * kBM / seg_len;
    const long long tiles = (segs + per_tile - 1) / per_tile * ((s.Co + bn - 1) / bn);
    if (tiles >= 2LL * sm_count()) {
      two = true;
      row_segs = per_tile;
    }
  }
  if (!two) {
    const long long m_seg = static_cast<long long>(s.batch) * OH *
                            ((OW + static_cast<int>(seg) - 1) / static_cast<int>(seg)) * seg;
    two = use_two_halves(bn, num_kb, m_seg, (s.Co + bn - 1) / bn);
  }
  CUtensorMap ma, mb;
  cuuint64_t da[4] = {static_cast<cuuint64_t>(s.Ci), static_cast<cuuint64_t>(s.W),
                      static_cast<cuuint64_t>(s.H),
                      static_cast<cuuint64_t>(s.batch)};
  cuuint64_t sa[3] = {static_cast<cuuint64_t>(s.Ci) * 2,
                      static_cast<cuuint64_t>(s.W) * s.Ci * 2,
                      static_cast<cuuint64_t>(s.H) * s.W * s.Ci * 2};
  cuuint32_t ba[4] = {kBK, row_segs ? static_cast<cuuint32_t>(seg_len) : seg, 1, 1};
  cuuint64_t db[3] = {static_cast<cuuint64_t>(s.Ci), static_cast<cuuint64_t>(taps),
                      static_cast<cuuint64_t>(s.Co)};
  cuuint64_t sb[2] = {static_cast<cuuint64_t>(s.Ci) * 2,
                      static_cast<cuuint64_t>(taps) * s.Ci * 2};
  cuuint32_t bb[3] = {kBK, 1, static_cast<cuuint32_t>(bn)};
  // Output map (NHWC y) for the TMA-store epilogue: one pixel segment of
  // one output row, 64 channels. Pixels past OW are not written.
  CUtensorMap mc;
  cuuint64_t dc[4] = {static_cast<cuuint64_t>(s.Co), static_cast<cuuint64_t>(OW),
                      static_cast<cuuint64_t>(OH),
                      static_cast<cuuint64_t>(s.batch)};
  cuuint64_t sc[3] = {static_cast<cuuint64_t>(epi.ldo) * 2,
                      static_cast<cuuint64_t>(OW) * epi.ldo * 2,
                      static_cast<cuuint64_t>(OH) * OW * epi.ldo * 2};
  cuuint32_t bc[4] = {64, row_segs ? 16u : seg, 1, 1};
  if (!encode(&ma, x, 4, da, sa, ba) || !encode(&mb, w, 3, db, sb, bb) ||
      !encode(&mc, epi.out, 4, dc, sc, bc))
    return cudaErrorInvalidValue;
  Args g{};
  g.seg_log2 = seg_log2;
  g.row_segs = row_segs;
  g.seg_len = seg_len ? seg_len : 16;
  g.seg_parts = seg_len ? OW / seg_len : 1;
  g.Wseg = (OW + static_cast<int>(seg) - 1) / static_cast<int>(seg);
  g.OH = OH;
  g.OW = OW;
  g.batch = s.batch;
  g.M = s.batch * OH * g.Wseg * static_cast<int>(seg);
  g.N = s.Co;
  g.kb_per_tap = (s.Ci + kBK - 1) / kBK;
  g.num_kb = g.kb_per_tap * taps;
  g.KW = s.KW;
  g.pad_h = s.pad_h;
  g.pad_w = s.pad_w;
  const int bm = two ? 2 * kBM : kBM;
  g.mt = row_segs ? (s.batch * OH * g.seg_parts + row_segs - 1) / row_segs
                  : (g.M + bm - 1) / bm;
  g.nt = (s.Co + bn - 1) / bn;
  g.epi = epi;
  g.err = device_error_word();
  return dispatch_bn<true, kEpiStore>(bn, two, ma, mb, mc, g, stream);
}

namespace {
// The second conv of a fused DB tail (kEpiDbTail); null for a plain deconv.
struct DbTail {
  const float *w;    // fp32 [64][4]
  const half *bias;  // or null
  half *out;         // fp16 [batch][4 H][4 W]
  int act;
};

cudaError_t deconv_impl(const half *x, const half *wpacked, const half *bias_rep,
                        half *y, int batch, int H, int W, int Ci, int Co, int KH,
                        int KW, int act, const DbTail *tail, cudaStream_t stream) {
  if (batch <= 0 || H <= 0 || W <= 0)
    return cudaSuccess;
  if (tail && (Co != 64 || KH != 2 || KW != 2 || !tail->w || !tail->out ||
               (reinterpret_cast<uintptr_t>(tail->out) & 3)))
    return cudaErrorInvalidValue;
  if (tail)
    y = tail->out; // the 64-channel map is not written; the store map goes unused
  const int N = KH * KW * Co;
  if (Co % 64 || Ci % 8 || !aligned16(x) || !aligned16(wpacked) ||
      !aligned16(y) || (bias_rep && !aligned16(bias_rep)))
    return cudaErrorInvalidValue;
  // N is a multiple of 64, so the tile (256, 128 or 64 columns) and each
  // 64-column store chunk cover whole taps' channel blocks.
  int bn = pick_bn(N);
  const int seg_log2 = W % 32 == 0 ? 5 : 4;
  const cuuint32_t seg = 1u << seg_log2;
  // One k-block per tile (Ci <= 64 in the DB head): the epilogue, not the
  // tensor core, sets the pace. With enough tiles, 256-row x 128-column
  // tiles put 8 epilogue warps on a double-buffered accumulator instead of
  // 4 warps on 128-row x 256-column tiles.
  const long long m_rows = static_cast<long long>(batch) * H *
                           ((W + static_cast<int>(seg) - 1) / static_cast<int>(seg)) * seg;
  const bool two = N % 128 == 0 && (Ci + kBK - 1) / kBK <= 2 &&
                   (m_rows + 2 * kBM - 1) / (2 * kBM) * (N / 128) >= 2LL * sm_count();
  if (two)
    bn = 128;
  CUtensorMap ma, mb, mc;
  cuuint64_t da[4] = {static_cast<cuuint64_t>(Ci), static_cast<cuuint64_t>(W),
                      static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(batch)};
  cuuint64_t sa[3] = {static_cast<cuuint64_t>(Ci) * 2, static_cast<cuuint64_t>(W) * Ci * 2,
                      static_cast<cuuint64_t>(H) * W * Ci * 2};
  cuuint32_t ba[4] = {kBK, seg, 1, 1};
  cuuint64_t db[3] = {static_cast<cuuint64_t>(Ci), 1, static_cast<cuuint64_t>(N)};
  cuuint64_t sb[2] = {static_cast<cuuint64_t>(Ci) * 2, static_cast<cuuint64_t>(Ci) * 2};
  cuuint32_t bb[3] = {kBK, 1, static_cast<cuuint32_t>(bn)};
  // Output y [batch][H*KH][W*KW][Co] seen as (co, b, w, a, n*H + h).
  const cuuint64_t ow = static_cast<cuuint64_t>(W) * KW;
  cuuint64_t dc[5] = {static_cast<cuuint64_t>(Co), static_cast<cuuint64_t>(KW),
                      static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(KH),
                      static_cast<cuuint64_t>(batch) * H};
  cuuint64_t scs[4] = {static_cast<cuuint64_t>(Co) * 2,
                       static_cast<cuuint64_t>(KW) * Co * 2, ow * Co * 2,
                       static_cast<cuuint64_t>(KH) * ow * Co * 2};
  cuuint32_t bc[5] = {64, 1, seg, 1, 1};
  if (!encode(&ma, x, 4, da, sa, ba) || !encode(&mb, wpacked, 3, db, sb, bb) ||
      !encode(&mc, y, 5, dc, scs, bc))
    return cudaErrorInvalidValue;
  Args g{};
  if (!tail && W % static_cast<int>(seg) == 0 && static_cast<long long>(batch) * H * W <= 0x7fffffffLL) {
    // No segment padding: the tiles' pixel rows are consecutive rows of
    // [pixels][Ci]; load them as 128-row boxes.
    cuuint64_t pa[2] = {static_cast<cuuint64_t>(Ci), static_cast<cuuint64_t>(batch) * H * W};
    cuuint64_t psa[1] = {static_cast<cuuint64_t>(Ci) * 2};
    cuuint32_t pba[2] = {kBK, kBM};
    if (!encode(&ma, x, 2, pa, psa, pba))
      return cudaErrorInvalidValue;
    g.plain_a = 1;
  }
  g.seg_log2 = seg_log2;
  g.Wseg = (W + static_cast<int>(seg) - 1) / static_cast<int>(seg);
  g.OH = H;
  g.OW = W;
  g.batch = batch;
  g.M = batch * H * g.Wseg * static_cast<int>(seg);
  g.N = N;
  g.kb_per_tap = (Ci + kBK - 1) / kBK;
  g.num_kb = g.kb_per_tap;
  g.KW = 1;
  g.mt = (g.M + (two ? 2 * kBM : kBM) - 1) / (two ? 2 * kBM : kBM);
  g.nt = (N + bn - 1) / bn;
  g.epi.bias = bias_rep;
  g.epi.out = y;
  g.epi.ldo = Co;
  g.epi.act = act;
  g.dec_co = Co;
  g.dec_kw = KW;
  g.err = device_error_word();
  if (tail) {
    // A pointwise GEMM over the input pixels: plain 2-D operand maps (the
    // pixel-segment maps above only serve the strided stores of a plain
    // deconv, which the fused tail does not make).
    const long long pixels = static_cast<long long>(batch) * H * W;
    if (pixels > 0x7fffffffLL)
      return cudaErrorInvalidValue;
    const int bt = two ? 128 : 256;
    cuuint64_t pa[2] = {static_cast<cuuint64_t>(Ci), static_cast<cuuint64_t>(pixels)};
    cuuint64_t psa[1] = {static_cast<cuuint64_t>(Ci) * 2};
    cuuint32_t pba[2] = {kBK, kBM};
    cuuint64_t pb[2] = {static_cast<cuuint64_t>(Ci), static_cast<cuuint64_t>(N)};
    cuuint64_t psb[1] = {static_cast<cuuint64_t>(Ci) * 2};
    cuuint32_t pbb[2] = {kBK, static_cast<cuuint32_t>(bt)};
    CUtensorMap pma, pmb;
    if (!encode(&pma, x, 2, pa, psa, pba) || !encode(&pmb, wpacked, 2, pb, psb, pbb))
      return cudaErrorInvalidValue;
    g.M = static_cast<int>(pixels);
    g.mt = (g.M + (two ? 2 * kBM : kBM) - 1) / (two ? 2 * kBM : kBM);
    g.nt = N / bt;
    g.tail_w = tail->w;
    g.tail_bias = tail->bias;
    g.tail_out = tail->out;
    g.tail_act = tail->act;
    if (two)
      return act == kActRelu ? launch<128, false, kEpiDbTail, kActRelu, 2>(pma, pmb, pma, g, stream)
                             : launch<128, false, kEpiDbTail, -1, 2>(pma, pmb, pma, g, stream);
    return act == kActRelu ? launch<256, false, kEpiDbTail, kActRelu>(pma, pmb, pma, g, stream)
                           : launch<256, false, kEpiDbTail, -1>(pma, pmb, pma, g, stream);
  }
  if (two)
    return act == kActRelu ? launch<128, true, kEpiDeconv, kActRelu, 2>(ma, mb, mc, g, stream)
                           : launch<128, true, kEpiDeconv, -1, 2>(ma, mb, mc, g, stream);
  switch (bn) {
  case 64:
    return act == kActRelu ? launch<64, true, kEpiDeconv, kActRelu>(ma, mb, mc, g, stream)
                           : launch<64, true, kEpiDeconv, -1>(ma, mb, mc, g, stream);
  case 128:
    return act == kActRelu ? launch<128, true, kEpiDeconv, kActRelu>(ma, mb, mc, g, stream)
                           : launch<128, true, kEpiDeconv, -1>(ma, mb, mc, g, stream);
  default:
    return act == kActRelu ? launch<256, true, kEpiDeconv, kActRelu>(ma, mb, mc, g, stream)
                           : launch<256, true, kEpiDeconv, -1>(ma, mb, mc, g, stream);
  }
}

__global__ void widen_kernel(const half *__restrict__ src, float *__restrict__ dst, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n)
    dst[i] = __half2float(src[i]);
}
} // namespace

cudaError_t tc_deconv(const half *x, const half *wpacked, const half *bias_rep,
                      half *y, int batch, int H, int W, int Ci, int Co, int KH,
                      int KW, int act, cudaStream_t stream) {
  return deconv_impl(x, wpacked, bias_rep, y, batch, H, W, Ci, Co, KH, KW, act, nullptr, stream);
}

cudaError_t tc_deconv_db_tail(const half *x, const half *wpacked, const half *bias_rep, int act,
                              const float *w2, const half *bias2, int act2, half *y2, int batch,
                              int H, int W, int Ci, cudaStream_t stream) {
  const DbTail tail{w2, bias2, y2, act2};
  return deconv_impl(x, wpacked, bias_rep, nullptr, batch, H, W, Ci, 64, 2, 2, act, &tail, stream);
}

cudaError_t widen_f16(const half *src, float *dst, int n, cudaStream_t stream) {
  if (n <= 0)
    return cudaSuccess;
  widen_kernel<<<(n + 255) / 256, 256, 0, stream>>>(src, dst, n);
  return cudaGetLastError();
}

cudaError_t tc_vocab_partials(const half *hidden, int rows, int H,
                              const half *wt, const half *bias, int V,
                              float *part_max, int *part_id, float *part_sum,
                              int calc_prob, cudaStream_t stream,
                              int *err_word) {
  if (rows <= 0)
    return cudaSuccess;
  if (H <= 0 || H % 8 || V <= 0 || !aligned16(hidden) || !aligned16(wt) ||
      !bias || !part_max || !part_id || !part_sum)
    return cudaErrorInvalidValue;
  CUtensorMap ma, mb;
  cuuint64_t da[2] = {static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(rows)};
  cuuint64_t sa[1] = {static_cast<cuuint64_t>(H) * 2};
  cuuint32_t ba[2] = {kBK, kBM};
  cuuint64_t db[2] = {static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(V)};
  cuuint32_t bb[2] = {kBK, 256};
  if (!encode(&ma, hidden, 2, da, sa, ba) || !encode(&mb, wt, 2, db, sa, bb))
    return cudaErrorInvalidValue;
  Args g{};
  g.M = rows;
  g.N = V;
  g.num_kb = (H + kBK - 1) / kBK;
  g.kb_per_tap = g.num_kb;
  g.KW = 1;
  g.mt = (rows + kBM - 1) / kBM;
  g.nt = vocab_tiles(V);
  g.Wseg = g.OH = g.OW = g.batch = 1;
  g.seg_log2 = 4;
  g.epi.bias = bias;
  g.part_max = part_max;
  g.part_id = part_id;
  g.part_sum = part_sum;
  g.part_ld = rows;
  g.calc_prob = calc_prob;
  g.err = err_word ? err_word : device_error_word();
  return launch<256, false, kEpiVocab, 0>(ma, mb, ma, g, stream);
}

} // namespace pb2
