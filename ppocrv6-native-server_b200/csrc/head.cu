// CTC head kernels: row argmax + softmax-max over fp16 logits, the merge of
// the tensor-core vocabulary partials, the greedy CTC collapse on device, the
// vocabulary weight transpose and the selected-class probability.
//
// Reference semantics (ppocrv6-native-server):
//   argmax / prob  native/src/kernels/classifier.cu:270-368, 456-515
//                  (ties -> lowest id, prob = 1 / sum __expf(l - max),
//                  per-tile sums rescaled by __expf(tile_max - row_max))
//   collapse       native/src/recognition/ctc_decode.cpp:7-51 (skip id equal
//                  to the previous id, then skip blank; score = sequential
//                  float mean of the kept probabilities, 0 if none kept)
//   selected class classifier.cu:111-143
#include "kernels.h"
#include "ptx.cuh"
#include <cfloat>
#include <climits>

namespace pb2 {
namespace {

// Row argmax / softmax-max over fp16 logits, one block per row, two
// passes: (1) the row max with packed fp16 max instructions (exact: fp16 ->
// fp32 is exact, so the fp16 max is the fp32 max); (2) sum exp(l - max) as
// ex2(l*log2e - max*log2e) on the special-function unit, and the lowest
// column holding the max (the argmax, ties -> lowest id), found by checking
// each 8-value vector's packed max against it. Rows of an odd vocabulary
// start at any 2-byte offset: the up to 7 logits before a row's first
// 16-byte boundary and after its last whole vector are handled one per
// thread.
constexpr int kArgmaxThreads = 128;

__device__ __forceinline__ half2 vec_max(const uint4 &u) {
  const half2 a = __hmax2(*reinterpret_cast<const half2 *>(&u.x),
                          *reinterpret_cast<const half2 *>(&u.y));
  const half2 b = __hmax2(*reinterpret_cast<const half2 *>(&u.z),
                          *reinterpret_cast<const half2 *>(&u.w));
  return __hmax2(a, b);
}

// The two passes over one row: elements [0, head) at hs[k], whole vectors
// vp[0..nvec) covering elements [head, head + 8*nvec), elements
// [head + 8*nvec, V) at gt[k] (global row pointer).
template <int THREADS>
__device__ __forceinline__ void argmax_row(const half *hs, int head,
                                           const uint4 *vp, int nvec,
                                           const half *gt, int V,
                                           long long row, int *ids,
                                           float *prob, float *max_logit,
                                           int calc_prob) {
  __shared__ float red_f[THREADS / 32];
  __shared__ int red_i[THREADS / 32];
  __shared__ float row_max;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t_idx = head + (nvec << 3) + tid; // this thread's tail element

  // ---- pass 1: max
  const half neg = __ushort_as_half(0xFC00); // -inf
  half2 m2 = __halves2half2(neg, neg);
  if (tid < head)
    m2 = __hmax2(m2, __halves2half2(hs[tid], neg));
  int v = tid;
  for (; v + 3 * THREADS < nvec; v += 4 * THREADS) {
    const uint4 u0 = vp[v], u1 = vp[v + THREADS];
    const uint4 u2 = vp[v + 2 * THREADS], u3 = vp[v + 3 * THREADS];
    m2 = __hmax2(m2, __hmax2(__hmax2(vec_max(u0), vec_max(u1)), __hmax2(vec_max(u2), vec_max(u3))));
  }
  for (; v < nvec; v += THREADS)
    m2 = __hmax2(m2, vec_max(vp[v]));
  if (t_idx < V)
    m2 = __hmax2(m2, __halves2half2(gt[t_idx], neg));
  float m = fmaxf(__low2float(m2), __high2float(m2));
#pragma unroll
  for (int o = 16; o; o >>= 1)
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0)
    red_f[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float r = red_f[0];
    for (int w = 1; w < THREADS / 32; ++w)
      r = fmaxf(r, red_f[w]);
    row_max = r;
  }
  __syncthreads();
  const float M = row_max;
  const half Mh = __float2half_rn(M); // exact: M is an fp16 value
  const float mL = M * kLog2e;

  // ---- pass 2: sum of exponentials and the first column holding the max
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  int best = INT_MAX;
  auto one = [&](float l, int idx) {
    s[0] += ex2_ftz(fmaf(l, kLog2e, -mL));
    if (l == M && idx < best)
      best = idx;
  };
  if (tid < head)
    one(__half2float(hs[tid]), tid);
  auto vec = [&](const uint4 &u, int vi) {
    if (calc_prob) {
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const half2 *>(&w[j]));
        s[j] += ex2_ftz(fmaf(f.x, kLog2e, -mL)) + ex2_ftz(fmaf(f.y, kLog2e, -mL));
      }
    }
    const half2 vm = vec_max(u);
    if (__heq(__high2half(vm), Mh) || __heq(__low2half(vm), Mh)) {
      const half *hv = reinterpret_cast<const half *>(&u);
      for (int j = 0; j < 8; ++j)
        if (__heq(hv[j], Mh)) {
          best = min(best, head + (vi << 3) + j);
          break;
        }
    }
  };
  v = tid;
  for (; v + 3 * THREADS < nvec; v += 4 * THREADS) {
    const uint4 u0 = vp[v], u1 = vp[v + THREADS];
    const uint4 u2 = vp[v + 2 * THREADS], u3 = vp[v + 3 * THREADS];
    vec(u0, v);
    vec(u1, v + THREADS);
    vec(u2, v + 2 * THREADS);
    vec(u3, v + 3 * THREADS);
  }
  for (; v < nvec; v += THREADS)
    vec(vp[v], v);
  if (t_idx < V)
    one(__half2float(gt[t_idx]), t_idx);
  float sum = (s[0] + s[1]) + (s[2] + s[3]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
  }
  __syncthreads();
  if (lane == 0) {
    red_f[warp] = sum;
    red_i[warp] = best;
  }
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    int b = INT_MAX;
    for (int w = 0; w < THREADS / 32; ++w) {
      t += red_f[w];
      b = min(b, red_i[w]);
    }
    ids[row] = b;
    max_logit[row] = M;
    prob[row] = calc_prob ? 1.f / t : 1.f;
  }
}

// Register form (unaligned logits base): 16-byte loads straight from
// global memory from the row's first 16-byte boundary.
__global__ void __launch_bounds__(kArgmaxThreads)
    logits_argmax_kernel(const half *__restrict__ logits, int V,
                         int *__restrict__ ids, float *__restrict__ prob,
                         float *__restrict__ max_logit, int calc_prob) {
  pdl_begin();
  const long long row = blockIdx.x;
  const half *lr = logits + row * V;
  const int head =
      min(V, static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(lr) & 15)) & 15) >> 1));
  const int nvec = (V - head) >> 3;
  argmax_row<kArgmaxThreads>(lr, head, reinterpret_cast<const uint4 *>(lr + head), nvec, lr,
                             V, row, ids, prob, max_logit, calc_prob);
}

__global__ void __launch_bounds__(256)
    vocab_merge_kernel(const float *__restrict__ pm, const int *__restrict__ pi,
                       const float *__restrict__ ps, int rows, int tiles,
                       int *__restrict__ ids, float *__restrict__ prob,
                       float *__restrict__ max_logit, int calc_prob) {
  pdl_begin();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows)
    return;
  float m = -FLT_MAX;
  int id = INT_MAX;
  for (int t = 0; t < tiles; ++t) {
    const float v = pm[static_cast<long long>(t) * rows + row];
    const int i = pi[static_cast<long long>(t) * rows + row];
    if (v > m || (v == m && i < id)) {
      m = v;
      id = i;
    }
  }
  float s = 0.f;
  if (calc_prob)
    for (int t = 0; t < tiles; ++t) {
      const float ts = ps[static_cast<long long>(t) * rows + row];
      s += ts == 0.f
               ? 0.f
               : ts * __expf(pm[static_cast<long long>(t) * rows + row] - m);
    }
  ids[row] = id;
  max_logit[row] = m;
  prob[row] = calc_prob ? 1.f / s : 1.f;
}

__global__ void __launch_bounds__(256)
    ctc_collapse_kernel(const int *__restrict__ ids,
                        const float *__restrict__ probs, int lines, int T,
                        int blank, int *__restrict__ out_ids,
                        int *__restrict__ out_len,
                        float *__restrict__ out_score) {
  pdl_begin();
  const int line = blockIdx.x * blockDim.x + threadIdx.x;
  if (line >= lines)
    return;
  const int *row = ids + static_cast<long long>(line) * T;
  const float *pr = probs ? probs + static_cast<long long>(line) * T : nullptr;
  int *dst = out_ids + static_cast<long long>(line) * T;
  int prev = -1, count = 0;
  float sum = 0.f;
  for (int t = 0; t < T; ++t) {
    const int id = row[t];
    if (id == prev)
      continue;
    prev = id;
    if (id == blank)
      continue;
    dst[count++] = id;
    sum += pr ? pr[t] : 1.0f;
  }
  for (int t = count; t < T; ++t)
    dst[t] = -1;
  out_len[line] = count;
  out_score[line] = count ? sum / static_cast<float>(count) : 0.f;
}

__global__ void __launch_bounds__(256)
    selected_class_kernel(const half *__restrict__ hidden,
                          const half *__restrict__ w,
                          const half *__restrict__ bias,
                          const float *__restrict__ max_logits,
                          float *__restrict__ out, int rows, int H, int V,
                          int cls) {
  pdl_begin();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows)
    return;
  float v = lane == 0 ? __half2float(bias[cls]) : 0.f;
  for (int h = lane; h < H; h += 32)
    v += __half2float(hidden[static_cast<long long>(row) * H + h]) *
         __half2float(w[static_cast<long long>(h) * V + cls]);
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) {
    const float ratio = __expf(fminf(v - max_logits[row], 0.f));
    out[row] = ratio / (1.f + ratio);
  }
}

// Register-resident row spans: columns [c0, c1) of one row (lr = row
// pointer) held by a block of THREADS threads as up to THREADS x VPT
// 16-byte vectors, every load issued before any arithmetic; the up to 7
// columns before the first 16-byte boundary and after the last whole vector
// are one per thread. Padding vector lanes hold -inf.
// A span's loads in flight: whole 16-byte vectors in u[], the head and tail
// columns one per thread.
template <int VPT>
struct SpanRegs {
  uint4 u[VPT];
  float xh, xt;
  int head, nvec, t0;
};

template <int THREADS, int VPT>
__device__ __forceinline__ void load_span(SpanRegs<VPT> &r, const half *__restrict__ lr,
                                          int c0, int c1) {
  const int tid = threadIdx.x;
  const int lead = static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(lr + c0) & 15)) & 15) >> 1);
  r.head = max(0, min(c1 - c0, lead));
  r.nvec = max(0, (c1 - c0 - r.head) >> 3);
  r.t0 = c0 + r.head + (r.nvec << 3); // first tail column
  const uint4 *vp = reinterpret_cast<const uint4 *>(lr + c0 + r.head);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = tid + k * THREADS;
    r.u[k] = v < r.nvec ? __ldcs(vp + v)
                        : make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u);
  }
  r.xh = tid < r.head ? __half2float(lr[c0 + tid]) : -INFINITY;
  r.xt = r.t0 + tid < c1 ? __half2float(lr[r.t0 + tid]) : -INFINITY;
}

// Single-barrier row reduction over register-resident spans. Each warp
// reduces its own columns to (warp max m_w, lowest column holding m_w,
// sum exp(l - m_w)); after one barrier warp 0 merges the warps:
// M = max m_w, id = lowest column among warps with m_w == M,
// sum = sum_w s_w * exp(m_w - M). Per logit: half a packed fp16 max, one
// conversion, half a packed fp32 FMA (l*log2e - m_w*log2e), one ex2 on the
// special-function unit and half a packed fp32 add; padding lanes hold -inf
// and contribute exp(-inf) = 0, so the vector loop has no bounds checks.
// Only lanes whose own max equals their warp's max scan their values for
// its first column. `slot` is THREADS/32 shared entries; a caller that
// reuses it for the next row alternates two sets (the barrier of row i+1
// orders warp 0's reads of row i before any write of row i+2).
struct WarpPart {
  float m, s;
  int id;
};

__device__ __forceinline__ void fadd2(float2 &acc, float2 v) {
  uint64_t d = (static_cast<uint64_t>(__float_as_uint(acc.y)) << 32) | __float_as_uint(acc.x);
  const uint64_t x = (static_cast<uint64_t>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
  asm("add.rn.f32x2 %0, %0, %1;" : "+l"(d) : "l"(x));
  acc.x = __uint_as_float(static_cast<uint32_t>(d));
  acc.y = __uint_as_float(static_cast<uint32_t>(d >> 32));
}

template <int THREADS, int VPT>
__device__ __forceinline__ void reduce_row_regs(const SpanRegs<VPT> &r, int V, int calc_prob,
                                                WarpPart *slot, long long row, int *ids,
                                                float *prob, float *max_logit) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  half2 m2 = vec_max(r.u[0]);
#pragma unroll
  for (int k = 1; k < VPT; ++k)
    m2 = __hmax2(m2, vec_max(r.u[k]));
  const float mt = fmaxf(fmaxf(__low2float(m2), __high2float(m2)), fmaxf(r.xh, r.xt));
  float mw = mt;
#pragma unroll
  for (int o = 16; o; o >>= 1)
    mw = fmaxf(mw, __shfl_xor_sync(0xffffffffu, mw, o));
  float sw = 0.f;
  if (calc_prob) {
    // A warp without columns has m_w = -inf: shift by 0 so every term is
    // exp(-inf) = 0 rather than NaN.
    const float mL = mw == -INFINITY ? 0.f : mw * kLog2e;
    const float2 l2 = make_float2(kLog2e, kLog2e);
    float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const uint32_t w[4] = {r.u[k].x, r.u[k].y, r.u[k].z, r.u[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 t = make_float2(-mL, -mL);
        ffma2(t, __half22float2(*reinterpret_cast<const half2 *>(&w[j])), l2);
        fadd2(acc[j & 1], make_float2(ex2_ftz(t.x), ex2_ftz(t.y)));
      }
    }
    sw = ((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y)) +
         (ex2_ftz(fmaf(r.xh, kLog2e, -mL)) + ex2_ftz(fmaf(r.xt, kLog2e, -mL)));
#pragma unroll
    for (int o = 16; o; o >>= 1)
      sw += __shfl_xor_sync(0xffffffffu, sw, o);
  }
  // Lowest column holding the warp max: head column, then the vectors in
  // column order, then the tail column of this thread.
  int best = INT_MAX;
  if (mt == mw && mw != -INFINITY) {
    const half Mh = __float2half_rn(mw); // exact: mw is an fp16 value
    // Compile-time indices only (r.u stays in registers).
    if (r.xt == mw)
      best = r.t0 + tid;
#pragma unroll
    for (int k = VPT - 1; k >= 0; --k) {
      const half *hv = reinterpret_cast<const half *>(&r.u[k]);
#pragma unroll
      for (int j = 7; j >= 0; --j)
        if (__heq(hv[j], Mh))
          best = r.head + ((tid + k * THREADS) << 3) + j;
    }
    if (r.xh == mw)
      best = tid;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1)
    best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0)
    slot[warp] = {mw, sw, best};
  __syncthreads();
  if (warp == 0) {
    constexpr int NW = THREADS / 32;
    const WarpPart e = lane < NW ? slot[lane] : WarpPart{-INFINITY, 0.f, INT_MAX};
    float M = e.m;
#pragma unroll
    for (int o = 16; o; o >>= 1)
      M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    int b = e.m == M ? e.id : INT_MAX;
    float t = e.s == 0.f ? 0.f : e.s * ex2_ftz((e.m - M) * kLog2e);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      b = min(b, __shfl_xor_sync(0xffffffffu, b, o));
      t += __shfl_xor_sync(0xffffffffu, t, o);
    }
    if (lane == 0) {
      ids[row] = b;
      max_logit[row] = M;
      prob[row] = calc_prob ? 1.f / t : 1.f;
    }
  }
}

// Row form: one block per row, the whole row in registers (V <= 8 x THREADS
// x VPT - 8), one barrier.
template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS)
    logits_argmax_row_kernel(const half *__restrict__ logits, int V,
                             int *__restrict__ ids, float *__restrict__ prob,
                             float *__restrict__ max_logit, int calc_prob) {
  pdl_begin();
  __shared__ WarpPart slot[THREADS / 32];
  const long long row = blockIdx.x;
  SpanRegs<VPT> r;
  load_span<THREADS, VPT>(r, logits + row * V, 0, V);
  reduce_row_regs<THREADS, VPT>(r, V, calc_prob, slot, row, ids, prob, max_logit);
}




} // namespace

cudaError_t logits_argmax_prob(const half *logits, int rows, int V, int *ids,
                               float *prob, float *max_logit, int calc_prob,
                               cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  if (V <= 0 || !ids || !prob || !max_logit)
    return cudaErrorInvalidValue;
  // Row form: the whole row in one block's registers, every load issued
  // before any arithmetic, one barrier (measured on B200 at BASELINE config
  // 1, 1,280 x 18,385 logits: 16.4 us by CUDA events, 13.3 us of device
  // time under ncu; the three-barrier form took 19.3 us, persistent forms
  // with the next row's loads in flight 20.7 us (two CTAs per SM, register
  // buffers) and 24.6 us (shared-memory ring of bulk copies), a row split
  // over a thread-block cluster 32.8 us, and computing a quarter of the
  // exponentials on the FMA pipe 17.9 us).
  auto row_form = [&](auto kernel, int threads) {
    launch_pdl(kernel, rows, threads, 0, s, logits, V, ids, prob, max_logit, calc_prob);
    return cudaGetLastError();
  };
  if (V <= 4088)
    return row_form(logits_argmax_row_kernel<256, 2>, 256);
  if (V <= 8184)
    return row_form(logits_argmax_row_kernel<256, 4>, 256);
  if (V <= 18424)
    return row_form(logits_argmax_row_kernel<256, 9>, 256);
  if (V <= 20472)
    return row_form(logits_argmax_row_kernel<512, 5>, 512);
  if (V <= 32760)
    return row_form(logits_argmax_row_kernel<512, 8>, 512);
  // Longer rows: 16-byte loads in a loop over the row (two passes).
  launch_pdl(logits_argmax_kernel, rows, kArgmaxThreads, 0, s, logits, V, ids, prob, max_logit,
      calc_prob);
  return cudaGetLastError();
}

namespace {
// Merge of the vocabulary partials with four threads per row: thread (r, q)
// of a 256-thread block takes row blockIdx.x * 64 + r and tiles q, q + 4,
// ... (loads coalesced across the block's 64 rows), then the four partial
// (max, lowest id) and, with the row max known, the four partial
// sum_t s_t * exp(m_t - max) are combined through shared memory. Same
// formula as vocab_merge_kernel; only the order of the fp32 sum differs.
__global__ void __launch_bounds__(256)
    vocab_merge4_kernel(const float *__restrict__ pm, const int *__restrict__ pi,
                        const float *__restrict__ ps, int rows, int tiles,
                        int *__restrict__ ids, float *__restrict__ prob,
                        float *__restrict__ max_logit, int calc_prob) {
  pdl_begin();
  __shared__ float sm[4][64];
  __shared__ int si[4][64];
  const int r = threadIdx.x & 63, q = threadIdx.x >> 6;
  const int row = blockIdx.x * 64 + r;
  float m = -FLT_MAX;
  int id = INT_MAX;
  if (row < rows)
    for (int t = q; t < tiles; t += 4) {
      const float v = pm[static_cast<long long>(t) * rows + row];
      const int i = pi[static_cast<long long>(t) * rows + row];
      if (v > m || (v == m && i < id)) {
        m = v;
        id = i;
      }
    }
  sm[q][r] = m;
  si[q][r] = id;
  __syncthreads();
  float M = sm[0][r];
  int I = si[0][r];
#pragma unroll
  for (int k = 1; k < 4; ++k)
    if (sm[k][r] > M || (sm[k][r] == M && si[k][r] < I)) {
      M = sm[k][r];
      I = si[k][r];
    }
  float s = 0.f;
  if (calc_prob && row < rows)
    for (int t = q; t < tiles; t += 4) {
      const float ts = ps[static_cast<long long>(t) * rows + row];
      s += ts == 0.f ? 0.f : ts * __expf(pm[static_cast<long long>(t) * rows + row] - M);
    }
  __syncthreads();
  sm[q][r] = s;
  __syncthreads();
  if (q == 0 && row < rows) {
    const float tot = (sm[0][r] + sm[1][r]) + (sm[2][r] + sm[3][r]);
    ids[row] = I;
    max_logit[row] = M;
    prob[row] = calc_prob ? 1.f / tot : 1.f;
  }
}
} // namespace

cudaError_t vocab_merge(const float *part_max, const int *part_id,
                        const float *part_sum, int rows, int tiles, int *ids,
                        float *prob, float *max_logit, int calc_prob,
                        cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  if (tiles >= 8) {
    launch_pdl(vocab_merge4_kernel, (rows + 63) / 64, 256, 0, s, part_max, part_id, part_sum, rows,
        tiles, ids, prob, max_logit, calc_prob);
    return cudaGetLastError();
  }
  launch_pdl(vocab_merge_kernel, (rows + 255) / 256, 256, 0, s, part_max, part_id, part_sum, rows,
      tiles, ids, prob, max_logit, calc_prob);
  return cudaGetLastError();
}

cudaError_t ctc_collapse(const int *ids, const float *probs, int lines, int T,
                         int blank, int *out_ids, int *out_len,
                         float *out_score, cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  if (T < 0 || !ids || !out_ids || !out_len || !out_score)
    return cudaErrorInvalidValue;
  launch_pdl(ctc_collapse_kernel, (lines + 255) / 256, 256, 0, s, ids, probs, lines, T, blank,
      out_ids, out_len, out_score);
  return cudaGetLastError();
}

cudaError_t pack_vocab_weight(const half *w, half *wt, int H, int V,
                              cudaStream_t s) {
  return transpose2d(w, wt, 1, H, V, s);
}

cudaError_t selected_class_vs_max(const half *hidden, const half *w,
                                  const half *bias, const float *max_logits,
                                  float *out, int rows, int H, int V,
                                  int class_id, cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  if (!hidden || !w || !bias || !max_logits || !out || H <= 0 || V <= 0 ||
      class_id < 0 || class_id >= V)
    return cudaErrorInvalidValue;
  launch_pdl(selected_class_kernel, (rows + 7) / 8, 256, 0, s, hidden, w, bias, max_logits, out,
      rows, H, V, class_id);
  return cudaGetLastError();
}

} // namespace pb2
