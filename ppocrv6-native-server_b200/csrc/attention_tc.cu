// SVTR mixing attention on the tensor cores (tcgen05 + TMEM), for the
// recognizer neck's short sequences (seq = 40, head_dim <= 16).
//
// Replaces the reference's attention chain (export.py lowers the ONNX graph
// to Runtime::matmul (q.k^T, cuBLAS strided-batched, FP32 compute),
// Runtime::softmax (reduce_kernel) and Runtime::matmul (P.v):
// native/src/compiled/runtime.cuh:1007-1024, 189-225) with one kernel and
// the same fp16 storage points: q' = round(q * scale), S = round(q'.k^T),
// P = round(softmax(S)), O = round(P.v).
//
// Work unit = (group of G = floor(128 / seq) lines, head). Its G * seq query
// rows (120 for seq 40) form the M = 128 rows of one UMMA tile, and its
// G * seq keys the N = 128 columns:
//  * the CTA's 128 threads (one per tile row) read their row's q, k and v
//    slices of this head as three aligned 48-byte windows (16-byte
//    cp.async copies into shared memory; the slices start at 30-byte
//    multiples), issued one unit ahead so that they land while the previous
//    unit computes, pick the head_dim values out (zero past head_dim),
//    scale and round q,
//    and write q' and k as the K-major A and B operands of S = q'.k^T
//    (M 128, N 128, K 16) and v transposed as the K-major B operand of
//    O = P.v (N 16, K 128), all in the canonical no-swizzle layout
//    (8-element K chunks as planes of 16-byte rows);
//  * one thread issues the S product into TMEM; each thread loads its row's
//    scores for its own line's keys (its warp loads the union window of the
//    lines its 32 rows cover), rounds them to fp16, and computes P with the
//    max-shifted exponentials on the SFU; P is written as the A operand of
//    the second product. Rows never see keys of another line: those blocks
//    of P are zero (written once at start and never touched);
//  * one thread issues the 8 K-steps of O = P.v into the first 16 columns
//    of the (then fully read) S accumulator; each thread loads its O row
//    from TMEM, rounds it and parks it in shared memory, and the CTA writes
//    the unit's head_dim-wide output column block row by row as 4-byte
//    words (eight consecutive threads per row), not as scattered halves.
// One unit at a time per CTA, three CTAs per SM (128 TMEM columns each);
// every mbarrier wait is bounded and its outcome is agreed block-wide, so a
// lost arrival makes the whole CTA record an error and leave together.
#include "kernels.h"
#include "ptx.cuh"

namespace pb2 {
namespace {

constexpr int kAttThreads = 128;
constexpr uint32_t kAPlane = 128 * 16;   // 128 rows x 8 fp16 (one K chunk)
constexpr uint32_t kVPlane = 16 * 16;    // 16 rows (head dims) x 8 keys
constexpr uint32_t kOffQ = 0;            // A of S: 2 planes
constexpr uint32_t kOffK = 2 * kAPlane;  // B of S: 2 planes
constexpr uint32_t kOffV = 4 * kAPlane;  // B of O: 16 planes of 256 B
constexpr uint32_t kOffP = kOffV + 16 * kVPlane; // A of O: 16 planes
constexpr uint32_t kOffRaw = kOffP + 16 * kAPlane; // 128 rows x 3 windows x 48 B
constexpr uint32_t kRawRow = 3 * 48;
constexpr uint32_t kOffOut = kOffRaw + 128 * kRawRow; // 128 rows x 16 fp16 of O
constexpr uint32_t kOffBar = kOffOut + 128 * 32;
constexpr uint32_t kTmemCols = 128;      // S: columns [0,128); O reuses [0,16)
constexpr int kAttCtasPerSm = 3;
// Dynamic shared memory per CTA (operands, raw windows, barriers).
constexpr size_t kAttSmem = kOffBar + 64;

struct AttArgs {
  const half *qkv; // [lines][seq][3][heads][dh]
  half *out;       // [lines][seq][heads][dh]
  int lines, seq, heads, dh;
  int G;      // lines per unit
  int units;  // ceil(lines / G) * heads
  float scale;
  int *err;
};

__device__ __forceinline__ uint64_t sdesc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

// 32 TMEM lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// 16-byte asynchronous global -> shared copy; bytes past src_bytes (0 or
// 16) are zero-filled and not read.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Issues the copies of tile row m's three 48-byte windows of unit u into its
// raw slot; returns the byte offsets of the head slices inside the windows.
__device__ __forceinline__ void fetch_windows(const AttArgs &g, int seq, int u, int m, uint32_t raw,
                                              uint32_t (&shift)[3]) {
  const int group = u / g.heads, h = u - group * g.heads;
  const int ell = m / seq, t = m - ell * seq;
  const int line = group * g.G + ell;
  const bool valid = m < g.G * seq && line < g.lines;
  // Element indices fit 32 bits (the launcher checks the tensor size).
  const uint32_t hd = static_cast<uint32_t>(g.heads * g.dh), width = 3 * hd;
  const uint32_t total = static_cast<uint32_t>(g.lines) * seq * width;
  const uint32_t row_e = (static_cast<uint32_t>(line) * seq + t) * width + h * g.dh;
#pragma unroll
  for (int sec = 0; sec < 3; ++sec) {
    const uint32_t e0 = row_e + sec * hd;
    const uint32_t a0 = e0 & ~7u; // 16-byte aligned element index
    shift[sec] = (e0 - a0) * 2;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      // Stay inside the tensor (the element count is a multiple of 8, so a
      // window chunk is wholly inside or wholly past the end).
      const bool in = valid && a0 + 8 * (c + 1) <= total;
      cp_async16(raw + sec * 48 + c * 16, in ? static_cast<const void *>(g.qkv + a0 + 8 * c) : g.qkv,
                 in ? 16u : 0u);
    }
  }
  cp_async_commit();
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

template <int SEQ>
__global__ void __launch_bounds__(kAttThreads, kAttCtasPerSm) attention_tc_kernel(const __grid_constant__ AttArgs g) {
  static_assert(SEQ % 8 == 0 && SEQ >= 32 && SEQ <= 64, "one or two lines per warp");
  constexpr int WIN = 2 * SEQ;    // a warp's 32 rows cover at most two lines
  extern __shared__ uint8_t att_smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(att_smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bar_s = reinterpret_cast<uint64_t *>(smem + kOffBar);
  uint64_t *bar_o = bar_s + 1;
  uint64_t *bar_drain = bar_s + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_s + 3);
  volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  pdl_launch_dependents();
  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_o, 1);
    mbar_init(bar_drain, 1);
    *abort = 0;
    fence_barrier_init();
  }
  // P is zero outside the diagonal (own-line) blocks, for good.
  for (uint32_t i = tid; i < 16 * kAPlane / 16; i += kAttThreads)
    sts_v4(sbase + kOffP + i * 16, make_uint4(0, 0, 0, 0));
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Nothing above touches global memory (programmatic dependent launch).
  pdl_wait();

  const int m = tid;                        // tile row (query) = key column
  const int rows = g.G * SEQ;
  const int ell = m / SEQ; // line within the unit
  // This warp's score window: the keys of the lines its rows belong to.
  const int w_lo = SEQ * ((warp * 32) / SEQ);
  const int w_hi = min(SEQ * ((warp * 32 + 31) / SEQ + 1), rows);
  const int own = SEQ * ell - w_lo;         // 0 or SEQ
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
  // Words of a head slice past head_dim are zero.
  uint32_t dmask[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    dmask[i] = (2 * i < g.dh ? 0xFFFFu : 0u) | (2 * i + 1 < g.dh ? 0xFFFF0000u : 0u);
  const uint32_t idesc_s = idesc_f16_f32(128, 128);
  const uint32_t idesc_o = idesc_f16_f32(128, 16);
  bool ok = true;
  int it = 0;
  const uint32_t raw = sbase + kOffRaw + static_cast<uint32_t>(m) * kRawRow;
  uint32_t shift[3] = {0, 0, 0};
  if (blockIdx.x < g.units)
    fetch_windows(g, SEQ, blockIdx.x, m, raw, shift);
  for (int u = blockIdx.x; u < g.units; u += gridDim.x, ++it) {
    const int group = u / g.heads, h = u - group * g.heads;
    const int line = group * g.G + ell;
    const bool valid = m < rows && line < g.lines;
    // ---- operands: q' and k rows (K-major), v transposed (K-major), from
    // this row's windows (its own copies only: no block barrier needed).
    cp_async_wait_all();
    const uint32_t sh0 = shift[0], sh1 = shift[1], sh2 = shift[2];
    uint32_t q[8], k[8], vw[8];
    {
      // head_dim halves starting `sh` bytes into a window, as 8 packed
      // words (zero past head_dim): 9 aligned 32-bit shared loads and a
      // 16-bit funnel shift when the slice starts mid-word.
      auto take = [&](uint32_t base, uint32_t sh, uint32_t (&w)[8]) {
        const uint32_t a = base + (sh & ~3u);
        uint32_t x[9];
#pragma unroll
        for (int i = 0; i < 9; ++i)
          x[i] = lds_u32(a + 4 * i);
        const uint32_t bits = (sh & 2u) * 8u;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          w[i] = __funnelshift_r(x[i], x[i + 1], bits) & (valid ? dmask[i] : 0u);
      };
      take(raw, sh0, q);
      take(raw + 48, sh1, k);
      take(raw + 96, sh2, vw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&q[j]));
        q[j] = pack2(f.x * g.scale, f.y * g.scale);
      }
    }
    // The next unit's windows load while this one computes.
    if (u + static_cast<int>(gridDim.x) < g.units)
      fetch_windows(g, SEQ, u + gridDim.x, m, raw, shift);
    const uint32_t row_off = static_cast<uint32_t>(m) * 16;
    sts_v4(sbase + kOffQ + row_off, make_uint4(q[0], q[1], q[2], q[3]));
    sts_v4(sbase + kOffQ + kAPlane + row_off, make_uint4(q[4], q[5], q[6], q[7]));
    sts_v4(sbase + kOffK + row_off, make_uint4(k[0], k[1], k[2], k[3]));
    sts_v4(sbase + kOffK + kAPlane + row_off, make_uint4(k[4], k[5], k[6], k[7]));
    {
      // v^T: head dim d is row d of the B operand, key m its K index.
      const uint32_t vb = sbase + kOffV + static_cast<uint32_t>(m >> 3) * kVPlane + static_cast<uint32_t>(m & 7) * 2;
#pragma unroll
      for (int d = 0; d < 16; ++d)
        asm volatile("st.shared.u16 [%0], %1;" ::"r"(vb + d * 16),
                     "h"(static_cast<uint16_t>(d & 1 ? vw[d >> 1] >> 16 : vw[d >> 1] & 0xFFFFu))
                     : "memory");
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- S = q'.k^T
    if (tid == 0) {
      tc_fence_after();
      umma_f16(tmem, sdesc_plain(sbase + kOffQ, kAPlane, 128), sdesc_plain(sbase + kOffK, kAPlane, 128), idesc_s,
               0);
      umma_commit(bar_s);
    }
    // One thread watches the barrier; the rest wait in the block barrier
    // (no issue slots spent spinning).
    if (tid == 0)
      ok = mbar_wait(bar_s, it & 1, abort);
    ok = __syncthreads_and(ok);
    if (!ok)
      break;
    tc_fence_after();
    // ---- P = round(softmax(round(S))) over the row's own line
    uint32_t r[WIN];
#pragma unroll
    for (int c = 0; c < WIN / 8; ++c)
      if (w_lo + 8 * c < w_hi)
        tmem_ld8(tmem + lane_base + static_cast<uint32_t>(w_lo + 8 * c), r + 8 * c);
    tmem_ld_wait();
    if (m < rows) {
      float s[SEQ];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < SEQ; ++j) {
        s[j] = round_half(__uint_as_float(own == 0 ? r[j] : r[SEQ + j]));
        mx = fmaxf(mx, s[j]);
      }
      // exp(s - max) = 2^(s*log2e - max*log2e), pairs of lanes per packed
      // fp32 FMA (each rounded once, as fmaf).
      const float mL = mx * kLog2e;
      float2 sum2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < SEQ; j += 2) {
        float2 a = make_float2(-mL, -mL);
        ffma2(a, make_float2(s[j], s[j + 1]), make_float2(kLog2e, kLog2e));
        s[j] = ex2_ftz(a.x);
        s[j + 1] = ex2_ftz(a.y);
        sum2.x += s[j];
        sum2.y += s[j + 1];
      }
      const float inv = 1.f / (sum2.x + sum2.y);
      const uint32_t pb = sbase + kOffP + static_cast<uint32_t>(SEQ * ell / 8) * kAPlane + row_off;
#pragma unroll
      for (int c = 0; c < SEQ / 8; ++c) {
        uint32_t pw[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 pp = make_float2(0.f, 0.f);
          ffma2(pp, make_float2(s[8 * c + 2 * e], s[8 * c + 2 * e + 1]), make_float2(inv, inv));
          pw[e] = pack2(pp.x, pp.y);
        }
        sts_v4(pb + c * kAPlane, make_uint4(pw[0], pw[1], pw[2], pw[3]));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- O = P.v
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_f16(tmem, sdesc_plain(sbase + kOffP + ks * 2 * kAPlane, kAPlane, 128),
                 sdesc_plain(sbase + kOffV + ks * 2 * kVPlane, kVPlane, 128), idesc_o, ks != 0);
      umma_commit(bar_o);
    }
    if (tid == 0)
      ok = mbar_wait(bar_o, it & 1, abort);
    ok = __syncthreads_and(ok);
    if (!ok)
      break;
    tc_fence_after();
    uint32_t o[16];
    tmem_ld16(tmem + lane_base, o);
    tmem_ld_wait();
    tc_fence_before();
    {
      const uint32_t ob = sbase + kOffOut + static_cast<uint32_t>(m) * 32;
      sts_v4(ob, make_uint4(pack2(__uint_as_float(o[0]), __uint_as_float(o[1])),
                            pack2(__uint_as_float(o[2]), __uint_as_float(o[3])),
                            pack2(__uint_as_float(o[4]), __uint_as_float(o[5])),
                            pack2(__uint_as_float(o[6]), __uint_as_float(o[7]))));
      sts_v4(ob + 16, make_uint4(pack2(__uint_as_float(o[8]), __uint_as_float(o[9])),
                                 pack2(__uint_as_float(o[10]), __uint_as_float(o[11])),
                                 pack2(__uint_as_float(o[12]), __uint_as_float(o[13])),
                                 pack2(__uint_as_float(o[14]), __uint_as_float(o[15]))));
    }
    __syncthreads();
    {
      // Output block of the unit: rows group*G*seq .. + rows, columns
      // [h*dh, h*dh + dh) of rows of heads*dh halves. Eight threads per row
      // write it as 32-bit words (a half at an unaligned start or end).
      const uint32_t hdw = static_cast<uint32_t>(g.heads * g.dh);
      const int row0 = group * g.G * SEQ;
      const int nrows = min(rows, g.lines * SEQ - row0);
      const int slot = tid & 7;
      // The 16 row passes are independent: all shared loads first, then
      // all stores.
      uint32_t wv[kAttThreads / 16];
      uint32_t *dstw[kAttThreads / 16];
#pragma unroll
      for (int i = 0; i < kAttThreads / 16; ++i) {
        const int rr = (tid >> 3) + i * (kAttThreads / 8);
        const uint32_t e0 = static_cast<uint32_t>(row0 + rr) * hdw + h * g.dh; // first element
        const int ld = static_cast<int>(e0 & 1u);            // a half before the first word
        const int j = ld + 2 * slot;
        const uint32_t ob = sbase + kOffOut + static_cast<uint32_t>(rr) * 32;
        wv[i] = (j & 1) ? (static_cast<uint32_t>(lds_u16(ob + 2 * j)) |
                           (static_cast<uint32_t>(lds_u16(ob + 2 * j + 2)) << 16))
                        : lds_u32(ob + 2 * j);
        dstw[i] = reinterpret_cast<uint32_t *>(reinterpret_cast<uint16_t *>(g.out) + e0 + j);
      }
#pragma unroll
      for (int i = 0; i < kAttThreads / 16; ++i) {
        const int rr = (tid >> 3) + i * (kAttThreads / 8);
        if (rr >= nrows)
          break;
        const uint32_t e0 = static_cast<uint32_t>(row0 + rr) * hdw + h * g.dh;
        const int ld = static_cast<int>(e0 & 1u);
        const int j = ld + 2 * slot;
        uint16_t *dst = reinterpret_cast<uint16_t *>(g.out) + e0;
        const uint32_t ob = sbase + kOffOut + static_cast<uint32_t>(rr) * 32;
        if (j + 1 < g.dh)
          *dstw[i] = wv[i];
        else if (j < g.dh)
          dst[j] = lds_u16(ob + 2 * j);
        if (slot == 0 && ld)
          dst[0] = lds_u16(ob);
      }
    }
  }
  cp_async_wait_all(); // no copy may land after the CTA is gone
  if (!ok) {
    // A wait ran out: record it, then let every issued product finish
    // (bounded) before the shared memory and TMEM go away.
    if (tid == 0) {
      *abort = 1;
      if (g.err)
        atomicCAS(g.err, 0, 41);
      umma_commit(bar_drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(bar_drain, 0) && clock64() - t0 < kWaitBudgetCycles) {
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    tmem_dealloc(tmem, kTmemCols);
}

} // namespace

bool attention_tc_supported(int seq, int dh) { return seq == 40 && dh >= 1 && dh <= 16; }

cudaError_t attention_tc(const half *qkv, half *out, int lines, int seq, int heads, int dh, float scale,
                         cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  // 16-byte window loads: the tensor is 16-byte aligned and (seq = 40) its
  // element count a multiple of 8, so no window straddles its end; output
  // words need a 4-byte aligned output.
  if (!attention_tc_supported(seq, dh) || heads <= 0 || (reinterpret_cast<uintptr_t>(qkv) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 3))
    return cudaErrorInvalidValue;
  // 32-bit element indices inside the kernel.
  if (static_cast<long long>(lines) * seq * 3 * heads * dh >= (1ll << 31))
    return cudaErrorInvalidValue;
  AttArgs a{};
  a.qkv = qkv;
  a.out = out;
  a.lines = lines;
  a.seq = seq;
  a.heads = heads;
  a.dh = dh;
  a.G = 128 / seq;
  a.units = (lines + a.G - 1) / a.G * heads;
  a.scale = scale;
  a.err = device_error_word();
  const size_t smem = kAttSmem + 1024; // + alignment slack
  cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<40>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess)
    return e;
  const int grid = std::min(a.units, kAttCtasPerSm * sm_count());
  launch_pdl(attention_tc_kernel<40>, grid, kAttThreads, smem, s, a);
  return cudaGetLastError();
}

} // namespace pb2
