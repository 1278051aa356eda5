// Batched matmul on the tensor cores for operands TMA cannot describe:
// Runtime::matmul with a computed right-hand side (the exporter's attention
// products q.k^T and P.v, native/src/compiled/runtime.cuh:1013-1024, which
// the reference runs as cuBLAS strided-batched GEMMs with FP32 compute).
// Their rows (k = head_dim = 15, n = seq = 40 halves) are not 16-byte
// multiples, so the operands are staged by SIMT loads instead of TMA.
//
// y[b] = round_fp16(A[b] . B[b]), A [m][k] and B [k][n] row-major, fp32
// accumulation in TMEM. CTA = 128 threads, one 128-row x NT-column output
// tile of one batch; K runs in chunks of 64:
//  * thread r copies row r of the A chunk (zero past m and k) and, for
//    r < NT, column r of the B chunk, into the canonical no-swizzle K-major
//    operand layouts (8-element K chunks as planes of 16-byte rows);
//  * thread 0 issues the chunk's four K = 16 UMMAs (M 128, N NT) and waits
//    for them (bounded); the others wait in the block barrier;
//  * after the last chunk each thread reads its accumulator row from TMEM,
//    rounds it to fp16 and stores it.
// k = 0 writes zeros.
#include "kernels.h"
#include "ptx.cuh"

namespace pb2 {
namespace {

constexpr int kMmThreads = 128;
constexpr int kMmKChunk = 64;
constexpr uint32_t kMmAPlane = 128 * 16; // 128 rows x 8 halves

struct MmArgs {
  const half *a, *b;
  half *y;
  int m, n, k;
  long long sa, sb, sy;
  int *err;
};

__device__ __forceinline__ uint64_t mm_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

__device__ __forceinline__ uint32_t mm_pack(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

template <int NT>
__global__ void __launch_bounds__(kMmThreads) matmul_tc_kernel(const __grid_constant__ MmArgs g) {
  constexpr uint32_t B_PLANE = NT * 16;
  constexpr uint32_t TMEM_COLS = NT < 32 ? 32 : NT;
  extern __shared__ uint8_t mm_smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(mm_smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sa = smem_u32(smem);                      // A: 8 planes
  const uint32_t sb = sa + 8 * kMmAPlane;                  // B: 8 planes
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + 8 * kMmAPlane + 8 * B_PLANE);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int batch = blockIdx.z, row0 = blockIdx.y * 128, col0 = blockIdx.x * NT;
  const half *A = g.a + batch * g.sa;
  const half *B = g.b + batch * g.sb;
  pdl_launch_dependents();
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Nothing above touches global memory (programmatic dependent launch).
  pdl_wait();
  const uint32_t idesc = idesc_f16_f32(128, NT);
  const int row = row0 + tid;
  const int col = col0 + tid;
  const uint16_t *a16 = reinterpret_cast<const uint16_t *>(A);
  const uint16_t *b16 = reinterpret_cast<const uint16_t *>(B);
  bool ok = true;
  int phase = 0;
  for (int k0 = 0; k0 < g.k; k0 += kMmKChunk, phase ^= 1) {
    // A chunk: row `row`, columns k0 .. k0+63.
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      uint16_t v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int kk = k0 + 8 * p + e;
        v[e] = row < g.m && kk < g.k ? __ldg(a16 + static_cast<long long>(row) * g.k + kk) : uint16_t(0);
      }
      sts_v4(sa + p * kMmAPlane + tid * 16,
             make_uint4(mm_pack(v[0], v[1]), mm_pack(v[2], v[3]), mm_pack(v[4], v[5]), mm_pack(v[6], v[7])));
    }
    // B chunk, transposed: column `col` (the N row of the operand).
    if (tid < NT) {
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        uint16_t v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int kk = k0 + 8 * p + e;
          v[e] = col < g.n && kk < g.k ? __ldg(b16 + static_cast<long long>(kk) * g.n + col) : uint16_t(0);
        }
        sts_v4(sb + p * B_PLANE + tid * 16,
               make_uint4(mm_pack(v[0], v[1]), mm_pack(v[2], v[3]), mm_pack(v[4], v[5]), mm_pack(v[6], v[7])));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int s = 0; s < 4; ++s)
        umma_f16(tmem, mm_desc(sa + 2 * s * kMmAPlane, kMmAPlane, 128), mm_desc(sb + 2 * s * B_PLANE, B_PLANE, 128),
                 idesc, (k0 > 0 || s > 0) ? 1u : 0u);
      umma_commit(bar);
      long long t0 = clock64();
      while (!mbar_try_wait(bar, phase)) {
        if (clock64() - t0 > kWaitBudgetCycles) {
          ok = false;
          break;
        }
      }
    }
    ok = __syncthreads_and(ok);
    if (!ok)
      break;
    tc_fence_after();
  }
  if (ok) {
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    uint16_t *y16 = reinterpret_cast<uint16_t *>(g.y + batch * g.sy);
#pragma unroll
    for (int c = 0; c < NT; c += 16) {
      uint32_t r[16];
      if (g.k > 0) {
        tmem_ld16(tmem + lane_base + c, r);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e)
          r[e] = 0;
      }
      if (row < g.m) {
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (col0 + c + e < g.n)
            y16[static_cast<long long>(row) * g.n + col0 + c + e] =
                __half_as_ushort(__float2half_rn(__uint_as_float(r[e])));
      }
    }
  } else if (tid == 0) {
    if (g.err)
      atomicCAS(g.err, 0, 51);
    // Let the issued products finish (bounded) before TMEM is freed.
    umma_commit(bar);
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, phase ^ 1) && clock64() - t0 < kWaitBudgetCycles) {
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    tmem_dealloc(tmem, TMEM_COLS);
}

template <int NT>
cudaError_t launch_mm(const MmArgs &a, int batches, cudaStream_t s) {
  constexpr int cols = NT < 32 ? 32 : NT;
  // Operands + barriers, raised so that no more CTAs share an SM than its
  // 512 TMEM columns serve at once.
  const size_t need = 8 * kMmAPlane + 8 * NT * 16 + 64 + 1024;
  const size_t per_sm = 228 * 1024;
  const int max_ctas = 512 / cols;
  const size_t floor_smem = max_ctas >= 16 ? 0 : per_sm / (max_ctas + 1) + 1024;
  const size_t smem = need > floor_smem ? need : floor_smem;
  cudaError_t e = cudaFuncSetAttribute(matmul_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess)
    return e;
  dim3 grid((a.n + NT - 1) / NT, (a.m + 127) / 128, batches);
  launch_pdl(matmul_tc_kernel<NT>, grid, kMmThreads, smem, s, a);
  return cudaGetLastError();
}

} // namespace

cudaError_t matmul_tc(const half *a, const half *b, half *y, int batches, int m, int n, int k, long long sa,
                      long long sb, long long sy, cudaStream_t s) {
  if (batches <= 0 || m <= 0 || n <= 0)
    return cudaSuccess;
  if (batches > 65535 || k < 0)
    return cudaErrorInvalidValue;
  MmArgs args{a, b, y, m, n, k, sa, sb, sy, device_error_word()};
  if (n <= 16)
    return launch_mm<16>(args, batches, s);
  if (n <= 32)
    return launch_mm<32>(args, batches, s);
  if (n <= 64)
    return launch_mm<64>(args, batches, s);
  return launch_mm<128>(args, batches, s);
}

} // namespace pb2
