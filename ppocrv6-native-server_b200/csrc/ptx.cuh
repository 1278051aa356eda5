// Inline-PTX primitives for sm_100a: mbarriers, TMA tile loads, tcgen05 (TMEM
// allocation, UMMA issue/commit, TMEM loads) and shared-memory descriptors.
//
// Every wait in this file is bounded: mbar_wait() gives up after a cycle budget
// and returns false so that the calling kernel can record an error, drain its
// own in-flight work and exit instead of spinning forever.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <utility>

namespace pb2 {

// ~2 s at 1.9 GHz. A legitimate wait in these kernels is at most one tile's
// K loop (tens of microseconds), so hitting this budget means a lost arrival.
constexpr long long kWaitBudgetCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Explicit shared-memory accesses by 32-bit shared address. Kernels that
// align their dynamic shared memory through integer arithmetic lose the
// address space on the pointer, and plain dereferences then compile to
// generic loads that wait on the long (L1TEX) scoreboard.
__device__ __forceinline__ uint16_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\t"
               "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\t"
               "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::
                   "r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\t"
               "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
               "selp.b32 %0, 1, 0, p;\n\t}"
               : "=r"(ok)
               : "r"(smem_u32(bar)), "r"(parity)
               : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete. Returns false if the
// cycle budget runs out or if *abort becomes non-zero (another role failed).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          volatile int *abort) {
  if (mbar_try_wait(bar, parity))
    return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort)
      return false;
    if (clock64() - t0 > kWaitBudgetCycles)
      return false;
  }
  return true;
}

// ------------------------------------------------ programmatic dependent launch
// Kernels of the layer path are launched with programmatic stream
// serialization (launch_pdl below, kept when a stream is captured into a
// CUDA graph): the next kernel's CTAs may be scheduled while this kernel's
// last CTAs run, so its launch and its global-memory-free prologue (barrier
// set-up, TMEM allocation, tensor-map prefetch) overlap them.
//  * pdl_wait(): blocks until every prerequisite grid has completed and its
//    memory operations are visible. Every kernel launched by launch_pdl calls
//    it in every CTA before its first global-memory access (read or write),
//    so completion of a kernel implies completion of all earlier ones.
//  * pdl_launch_dependents(): lets the dependent grid be scheduled once every
//    CTA of this grid has issued it (or exited). Safe at any point: the
//    dependent still waits for this grid's completion in pdl_wait().
// Both are no-ops for a grid launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// The two together, for kernels without a prologue to overlap.
__device__ __forceinline__ void pdl_begin() {
  pdl_launch_dependents();
  pdl_wait();
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args &&...args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- TMA loads
// Tiled bulk-tensor loads into this CTA's shared memory, completing on an
// mbarrier (complete_tx). Every load targets this CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
      "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
      "r"(c2), "r"(c3)
      : "memory");
}
// Untiled bulk copy global -> this CTA's shared memory, completing on an
// mbarrier. Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void *dst, const void *src,
                                          uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
               "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes),
               "r"(smem_u32(bar))
               : "memory");
}
// Tiled bulk-tensor stores from this CTA's shared memory (bulk-group
// completion). Out-of-range rows/columns of the box are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map,
                                             const void *src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group "
               "[%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map,
                                             const void *src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group "
               "[%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void tma_store_5d(const CUtensorMap *map,
                                             const void *src, int c0, int c1,
                                             int c2, int c3, int c4) {
  asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.tile.bulk_group "
               "[%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
               : "memory");
}
// Untiled bulk copy this CTA's shared memory -> global (bulk-group
// completion). Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store(void *dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
               "r"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's bulk groups still read smem.
template <int N> __device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Orders this thread's generic-proxy smem writes before async-proxy reads.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(slot)),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 in, fp32 acc).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc,
                                         uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\t"
               "setp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::
                   "r"(d_tmem),
               "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
               : "memory");
}
// Arrives once on `bar` when every previously issued tcgen05.mma of this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::"
               "cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 TMEM lanes x 16 consecutive 32-bit columns: lane i of the warp receives
// row (lane base + i), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
                 "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
                 "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                 "=r"(r[14]), "=r"(r[15])
               : "r"(taddr)
               : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 64 fp16 (128 B), 8-row swizzle atoms of
// 1024 B. SBO = 1024 B between 8-row groups; LBO is unused for this layout
// (encoded as 1); version field = 1 (sm_100); layout type 2 = SWIZZLE_128B.
// The tile base must be 1024-byte aligned; the K offset inside the 128-byte
// row is added to the start address (32 B per 16-element K step).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp16 A/B, fp32 accumulator, both
// operands K-major, dense. M in {64,128}, N a multiple of 16 up to 256.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                                   // D format: f32
         | (0u << 7) | (0u << 10)                    // A, B: f16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

__device__ __forceinline__ float round_half(float v) {
  return __half2float(__float2half_rn(v));
}

// Activation codes shared by every fused epilogue. 0..2 follow the reference
// runtime (bias only, ReLU, erf-GELU); 3..6 extend it for folded
// HardSigmoid*x, Sigmoid, x*Sigmoid and HardSigmoid chains.
enum Act : int {
  kActNone = 0,
  kActRelu = 1,
  kActGelu = 2,
  kActHardSwish = 3,
  kActSigmoid = 4,
  kActSwish = 5,
  kActHardSigmoid = 6,
};

__device__ __forceinline__ float apply_act(float x, int act);

// Compile-time activation (ACT >= 0) keeps unrolled epilogues small; ACT < 0
// falls back to the runtime switch.
template <int ACT>
__device__ __forceinline__ float act_t(float x, int act) {
  if constexpr (ACT < 0)
    return apply_act(x, act);
  else if constexpr (ACT == kActNone)
    return x;
  else if constexpr (ACT == kActRelu)
    return fmaxf(x, 0.f);
  else if constexpr (ACT == kActHardSwish)
    return x * fminf(1.f, fmaxf(0.f, __fmaf_rn(0.166666671634f, x, 0.5f)));
  else if constexpr (ACT == kActSwish)
    // Branch-free x * sigmoid(x) for the unrolled GEMM epilogues: hardware
    // exp2 and reciprocal (relative error ~1e-6, far below the fp16 output
    // rounding); x -> -inf gives x * 0 = -0.
    return __fdividef(x, 1.f + __expf(-x));
  else
    return apply_act(x, ACT);
}

__device__ __forceinline__ float apply_act(float x, int act) {
  switch (act) {
  case kActRelu:
    return fmaxf(x, 0.f);
  case kActGelu:
    return (x * (erff(x / 1.41421354f) + 1.f)) * 0.5f;
  case kActHardSwish: // HardSigmoid(alpha=1/6, beta=1/2) * x, one FMA
    return x * fminf(1.f, fmaxf(0.f, __fmaf_rn(0.166666671634f, x, 0.5f)));
  case kActSigmoid:
    return 1.f / (1.f + expf(-x));
  case kActSwish:
    return x * (1.f / (1.f + expf(-x)));
  case kActHardSigmoid:
    return fminf(1.f, fmaxf(0.f, __fmaf_rn(0.166666671634f, x, 0.5f)));
  default:
    return x;
  }
}

// Mixed-precision arithmetic (PTX ISA 8.6, sm_100): fp16 operands with an
// fp32 accumulator in one instruction. fp16 -> fp32 conversion is exact and
// the product of two fp16 values is exact in fp32, so fma2_h gives the same
// bits as fmaf(float(x), float(w), acc) and add2_h as acc + float(x).
// x and w hold two fp16 values each (low half, high half).
__device__ __forceinline__ void fma2_h(float &lo, float &hi, uint32_t x,
                                       uint32_t w) {
  asm("{.reg .f16 xl, xh, wl, wh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "mov.b32 {wl, wh}, %3;\n\t"
      "fma.rn.f32.f16 %0, xl, wl, %0;\n\t"
      "fma.rn.f32.f16 %1, xh, wh, %1;}"
      : "+f"(lo), "+f"(hi)
      : "r"(x), "r"(w));
}
__device__ __forceinline__ void add2_h(float &lo, float &hi, uint32_t x) {
  asm("{.reg .f16 xl, xh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "add.rn.f32.f16 %0, xl, %0;\n\t"
      "add.rn.f32.f16 %1, xh, %1;}"
      : "+f"(lo), "+f"(hi)
      : "r"(x));
}
// Packed fp32 pair FMA (PTX ISA 8.6, sm_100): acc.{x,y} = a.{x,y} * b.{x,y}
// + acc.{x,y}, each lane rounded once (the same bits as two fmaf calls).
__device__ __forceinline__ void ffma2(float2 &acc, float2 a, float2 b) {
  uint64_t d = (static_cast<uint64_t>(__float_as_uint(acc.y)) << 32) | __float_as_uint(acc.x);
  const uint64_t x = (static_cast<uint64_t>(__float_as_uint(a.y)) << 32) | __float_as_uint(a.x);
  const uint64_t y = (static_cast<uint64_t>(__float_as_uint(b.y)) << 32) | __float_as_uint(b.x);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(x), "l"(y));
  acc.x = __uint_as_float(static_cast<uint32_t>(d));
  acc.y = __uint_as_float(static_cast<uint32_t>(d >> 32));
}
// 2^x on the special-function unit (approximate, subnormal results flushed).
// exp(v - m) is computed as ex2(v * log2(e) - m * log2(e)).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

// Host: encodes an fp16 tiled tensor map (innermost dimension first, byte
// strides for dimensions 1..rank-1; out-of-range elements read as zero),
// 128-byte swizzled or unswizzled. False if the driver rejects it.
bool encode_fp16_map(CUtensorMap *m, const void *base, int rank,
                     const cuuint64_t *dims, const cuuint64_t *strides,
                     const cuuint32_t *box, bool swizzle128);

// Unsigned division by a run-time invariant for dividends below 2^31
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, m) + n) >> l.
// Kernels index their work items with 32-bit counters and these in place
// of 64-bit divisions (which compile to long instruction sequences).
struct FastDiv {
  uint32_t d = 1, m = 1, l = 0;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t div) : d(div) {
    l = 0;
    while ((1ull << l) < div)
      ++l;
    m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - div)) / div + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (__umulhi(n, m) + n) >> l;
  }
};

} // namespace pb2
