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
#include <cooperative_groups.h>
#include "ptx.cuh"
#include <algorithm>
#include <cfloat>
#include <climits>
#include <mutex>

namespace pb2 {
namespace {

// Row argmax / softmax-max over fp16 logits, one 128-thread block per row,
// two passes: (1) the row max with packed fp16 max instructions (exact:
// fp16 -> fp32 is exact, so the fp16 max is the fp32 max); (2) sum
// exp(l - max) as ex2(l*log2e - max*log2e) on the special-function unit,
// and the lowest column holding the max (the argmax, ties -> lowest id),
// found by checking each 8-value vector's packed max against it.
//
// The row is staged in shared memory by bulk copies (cp.async.bulk, 8 KB
// each, one mbarrier): the 16-byte-aligned span of the row (rows of an odd
// vocabulary start at any 2-byte offset), so a block has the whole 36 KB row
// in flight with one instruction per 8 KB. The up to 7 logits before the
// first aligned vector inside the span and after its end are handled one
// by one (the latter read from global memory).
constexpr int kArgmaxThreads = 128;
constexpr uint32_t kBulkChunk = 8192;

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
__device__ __forceinline__ void argmax_row(const half *hs, int head,
                                           const uint4 *vp, int nvec,
                                           const half *gt, int V,
                                           long long row, int *ids,
                                           float *prob, float *max_logit,
                                           int calc_prob) {
  __shared__ float red_f[kArgmaxThreads / 32];
  __shared__ int red_i[kArgmaxThreads / 32];
  __shared__ float row_max;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t_idx = head + (nvec << 3) + tid; // this thread's tail element

  // ---- pass 1: max
  const half neg = __ushort_as_half(0xFC00); // -inf
  half2 m2 = __halves2half2(neg, neg);
  if (tid < head)
    m2 = __hmax2(m2, __halves2half2(hs[tid], neg));
  int v = tid;
  for (; v + 3 * kArgmaxThreads < nvec; v += 4 * kArgmaxThreads) {
    const uint4 u0 = vp[v], u1 = vp[v + kArgmaxThreads];
    const uint4 u2 = vp[v + 2 * kArgmaxThreads], u3 = vp[v + 3 * kArgmaxThreads];
    m2 = __hmax2(m2, __hmax2(__hmax2(vec_max(u0), vec_max(u1)), __hmax2(vec_max(u2), vec_max(u3))));
  }
  for (; v < nvec; v += kArgmaxThreads)
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
    for (int w = 1; w < kArgmaxThreads / 32; ++w)
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
  for (; v + 3 * kArgmaxThreads < nvec; v += 4 * kArgmaxThreads) {
    const uint4 u0 = vp[v], u1 = vp[v + kArgmaxThreads];
    const uint4 u2 = vp[v + 2 * kArgmaxThreads], u3 = vp[v + 3 * kArgmaxThreads];
    vec(u0, v);
    vec(u1, v + kArgmaxThreads);
    vec(u2, v + 2 * kArgmaxThreads);
    vec(u3, v + 3 * kArgmaxThreads);
  }
  for (; v < nvec; v += kArgmaxThreads)
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
    for (int w = 0; w < kArgmaxThreads / 32; ++w) {
      t += red_f[w];
      b = min(b, red_i[w]);
    }
    ids[row] = b;
    max_logit[row] = M;
    prob[row] = calc_prob ? 1.f / t : 1.f;
  }
}

// Rows staged in shared memory (logits base 16-byte aligned). Persistent:
// a block walks rows blockIdx.x, blockIdx.x + gridDim.x, ... with two row
// buffers, the next row's bulk copies in flight while the current row is
// reduced.
struct RowSpan {
  uint64_t a0;     // first copied byte (16-byte aligned)
  uint32_t nbytes; // bytes copied (multiple of 16)
  int off;         // row element 0 sits at shared half index off
  int in_smem;     // row elements inside the copied span
};

__device__ __forceinline__ RowSpan row_span(long long row, int V) {
  RowSpan r;
  const uint64_t start_b = static_cast<uint64_t>(row) * V * 2;
  r.a0 = start_b & ~uint64_t(15);
  const uint64_t a1 = (start_b + 2ull * V) & ~uint64_t(15);
  r.nbytes = a1 > r.a0 ? static_cast<uint32_t>(a1 - r.a0) : 0;
  r.off = static_cast<int>((start_b - r.a0) >> 1);
  r.in_smem = static_cast<int>((a1 > start_b ? a1 - start_b : 0) >> 1);
  return r;
}

__global__ void __launch_bounds__(kArgmaxThreads)
    logits_argmax_bulk_kernel(const half *__restrict__ logits, int V, int rows,
                              uint32_t buf_bytes, int *__restrict__ ids,
                              float *__restrict__ prob,
                              float *__restrict__ max_logit, int calc_prob,
                              int *err) {
  extern __shared__ uint4 row_smem[];
  __shared__ uint64_t bar[2];
  __shared__ int failed;
  const char *base = reinterpret_cast<const char *>(logits);
  auto buf = [&](int b) {
    return reinterpret_cast<uint4 *>(reinterpret_cast<char *>(row_smem) + b * buf_bytes);
  };
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    failed = 0;
    fence_barrier_init();
  }
  __syncthreads();
  auto issue = [&](long long row, int b) {
    const RowSpan sp = row_span(row, V);
    if (!sp.nbytes)
      return;
    mbar_arrive_expect_tx(&bar[b], sp.nbytes);
    for (uint32_t o = 0; o < sp.nbytes; o += kBulkChunk)
      bulk_load(reinterpret_cast<char *>(buf(b)) + o, base + sp.a0 + o,
                min(kBulkChunk, sp.nbytes - o), &bar[b]);
  };
  long long row = blockIdx.x;
  if (threadIdx.x == 0 && row < rows)
    issue(row, 0);
  uint32_t uses0 = 0, uses1 = 0; // completed phases per buffer
  volatile int no_abort = 0;
  for (int k = 0; row < rows; ++k, row += gridDim.x) {
    const int b = k & 1;
    const long long next = row + gridDim.x;
    // The other buffer was last read by the previous iteration, which every
    // thread has left (barrier at the end of the loop body).
    if (threadIdx.x == 0 && next < rows)
      issue(next, b ^ 1);
    const RowSpan sp = row_span(row, V);
    bool ok = true;
    uint32_t &uses = b ? uses1 : uses0;
    if (sp.nbytes) {
      ok = mbar_wait(&bar[b], uses & 1, &no_abort);
      ++uses;
    }
    if (!ok)
      failed = 1;
    __syncthreads();
    if (failed) {
      // A bounded wait ran out: report, give this block's copies in flight
      // one more budget to land, and stop.
      if (threadIdx.x == 0) {
        if (err)
          atomicCAS(err, 0, 6);
        if (!ok)
          mbar_wait(&bar[b], (uses - 1) & 1, &no_abort);
        if (next < rows && row_span(next, V).nbytes)
          mbar_wait(&bar[b ^ 1], (b ? uses0 : uses1) & 1, &no_abort);
      }
      return;
    }
    const half *rs = reinterpret_cast<const half *>(buf(b)) + sp.off;
    const int head = min(sp.in_smem, sp.off ? 8 - sp.off : 0);
    const int nvec = (sp.in_smem - head) >> 3;
    argmax_row(rs, head, buf(b) + (sp.off ? 1 : 0), nvec, logits + row * V, V,
               row, ids, prob, max_logit, calc_prob);
    __syncthreads();
  }
}

// Register form (unaligned logits base): 16-byte loads straight from
// global memory from the row's first 16-byte boundary.
__global__ void __launch_bounds__(kArgmaxThreads)
    logits_argmax_kernel(const half *__restrict__ logits, int V,
                         int *__restrict__ ids, float *__restrict__ prob,
                         float *__restrict__ max_logit, int calc_prob) {
  const long long row = blockIdx.x;
  const half *lr = logits + row * V;
  const int head =
      min(V, static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(lr) & 15)) & 15) >> 1));
  const int nvec = (V - head) >> 3;
  argmax_row(lr, head, reinterpret_cast<const uint4 *>(lr + head), nvec, lr, V,
             row, ids, prob, max_logit, calc_prob);
}

__global__ void __launch_bounds__(256)
    vocab_merge_kernel(const float *__restrict__ pm, const int *__restrict__ pi,
                       const float *__restrict__ ps, int rows, int tiles,
                       int *__restrict__ ids, float *__restrict__ prob,
                       float *__restrict__ max_logit, int calc_prob) {
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

// Cluster form: a row is split over a thread-block cluster of P CTAs (P <=
// 8), each reducing a column range of at most 4 x 128 x 8 logits held in
// registers (every 16-byte load of the range is issued up front), to
// (max, lowest argmax, sum exp(l - max)); the cluster then merges the P
// partials through distributed shared memory in column order, so ties still
// resolve to the lowest id. No global scratch, one launch.
constexpr int kClusterThreads = 128;
constexpr int kClusterVpt = 4; // 16-byte vectors per thread

struct Partial {
  float m;
  float s;
  int id;
};

__global__ void __launch_bounds__(kClusterThreads)
    logits_argmax_cluster_kernel(const half *__restrict__ logits, int V,
                                 int chunk, int *__restrict__ ids,
                                 float *__restrict__ prob,
                                 float *__restrict__ max_logit, int calc_prob) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ Partial part;
  __shared__ float red_f[kClusterThreads / 32];
  __shared__ int red_i[kClusterThreads / 32];
  const int P = static_cast<int>(cluster.num_blocks());
  const int q = static_cast<int>(cluster.block_rank());
  const long long row = blockIdx.x / P;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = q * chunk;
  const int c1 = min(V, c0 + chunk);
  const half *lr = logits + row * V;
  // [c0, c1): head elements up to the first 16-byte boundary, whole vectors,
  // tail elements.
  const int lead = static_cast<int>(((16 - (reinterpret_cast<uintptr_t>(lr + c0) & 15)) & 15) >> 1);
  const int head = max(0, min(c1 - c0, lead));
  const int nvec = max(0, (c1 - c0 - head) >> 3);
  const int t0 = c0 + head + (nvec << 3); // first tail element
  const uint4 *vp = reinterpret_cast<const uint4 *>(lr + c0 + head);
  uint4 u[kClusterVpt];
#pragma unroll
  for (int k = 0; k < kClusterVpt; ++k) {
    const int v = tid + k * kClusterThreads;
    u[k] = v < nvec ? __ldcs(vp + v) : make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u);
  }
  const bool has_head = tid < head;
  const bool has_tail = t0 + tid < c1;
  const float xh = has_head ? __half2float(lr[c0 + tid]) : -INFINITY;
  const float xt = has_tail ? __half2float(lr[t0 + tid]) : -INFINITY;
  // pass 1: max (padding lanes hold -inf)
  half2 m2 = vec_max(u[0]);
#pragma unroll
  for (int k = 1; k < kClusterVpt; ++k)
    m2 = __hmax2(m2, vec_max(u[k]));
  float m = fmaxf(fmaxf(__low2float(m2), __high2float(m2)), fmaxf(xh, xt));
#pragma unroll
  for (int o = 16; o; o >>= 1)
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0)
    red_f[warp] = m;
  __syncthreads();
  float M = red_f[0];
#pragma unroll
  for (int w = 1; w < kClusterThreads / 32; ++w)
    M = fmaxf(M, red_f[w]);
  __syncthreads();
  // pass 2: sum of exponentials, first column holding the max
  const half Mh = __float2half_rn(M);
  const float mL = M * kLog2e;
  float sacc[4] = {0.f, 0.f, 0.f, 0.f};
  int best = INT_MAX;
  if (has_head) {
    sacc[0] += ex2_ftz(fmaf(xh, kLog2e, -mL));
    if (xh == M)
      best = c0 + tid;
  }
#pragma unroll
  for (int k = 0; k < kClusterVpt; ++k) {
    const int v = tid + k * kClusterThreads;
    if (v < nvec) {
      if (calc_prob) {
        const uint32_t w[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(*reinterpret_cast<const half2 *>(&w[j]));
          sacc[j] += ex2_ftz(fmaf(f.x, kLog2e, -mL)) + ex2_ftz(fmaf(f.y, kLog2e, -mL));
        }
      }
      const half2 vm = vec_max(u[k]);
      if (__heq(__high2half(vm), Mh) || __heq(__low2half(vm), Mh)) {
        const half *hv = reinterpret_cast<const half *>(&u[k]);
        for (int j = 0; j < 8; ++j)
          if (__heq(hv[j], Mh)) {
            best = min(best, c0 + head + (v << 3) + j);
            break;
          }
      }
    }
  }
  if (has_tail) {
    sacc[1] += ex2_ftz(fmaf(xt, kLog2e, -mL));
    if (xt == M)
      best = min(best, t0 + tid);
  }
  float sum = (sacc[0] + sacc[1]) + (sacc[2] + sacc[3]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
  }
  if (lane == 0) {
    red_f[warp] = sum;
    red_i[warp] = best;
  }
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    int b = INT_MAX;
    for (int w = 0; w < kClusterThreads / 32; ++w) {
      t += red_f[w];
      b = min(b, red_i[w]);
    }
    part.m = c1 > c0 ? M : -INFINITY;
    part.s = c1 > c0 && calc_prob ? t : 0.f;
    part.id = b;
  }
  cluster.sync(); // every CTA's partial is written
  if (q == 0 && tid == 0) {
    float gm = -INFINITY;
    int gid = INT_MAX;
    Partial ps[8];
    for (int r = 0; r < P; ++r) {
      ps[r] = *cluster.map_shared_rank(&part, r);
      if (ps[r].m > gm) { // ranks are in column order: ties keep the lower id
        gm = ps[r].m;
        gid = ps[r].id;
      }
    }
    float gs = 0.f;
    for (int r = 0; r < P; ++r)
      gs += ps[r].s == 0.f ? 0.f : ps[r].s * ex2_ftz((ps[r].m - gm) * kLog2e);
    ids[row] = gid;
    max_logit[row] = gm;
    prob[row] = calc_prob ? 1.f / gs : 1.f;
  }
  cluster.sync(); // rank 0 has read the partials before any CTA exits
}

} // namespace

cudaError_t logits_argmax_prob(const half *logits, int rows, int V, int *ids,
                               float *prob, float *max_logit, int calc_prob,
                               cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  if (V <= 0 || !ids || !prob || !max_logit)
    return cudaErrorInvalidValue;
  // Cluster form when a row fits P <= 8 CTAs' registers.
  const int per_cta = kClusterThreads * kClusterVpt * 8 - 8; // alignment slack
  const int P = (V + per_cta - 1) / per_cta;
  if (P <= 8 && static_cast<long long>(rows) * P < (1LL << 31)) {
    const int chunk = ((V + P - 1) / P + 7) & ~7;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(rows * P));
    cfg.blockDim = dim3(kClusterThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(P);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, logits_argmax_cluster_kernel, logits, V, chunk, ids,
                              prob, max_logit, calc_prob);
  }
  const size_t row_bytes = (2ull * V + 31) & ~size_t(15);
  if ((reinterpret_cast<uintptr_t>(logits) & 15) == 0 && 2 * row_bytes <= 200 * 1024) {
    static std::once_flag once[64];
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t attr = cudaSuccess;
    std::call_once(once[dev & 63], [&] {
      attr = cudaFuncSetAttribute(logits_argmax_bulk_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  200 * 1024);
    });
    if (attr != cudaSuccess)
      return attr;
    // Blocks per SM as shared memory allows (two row buffers each).
    const int per_sm = static_cast<int>(
        std::max<size_t>(1, std::min<size_t>(8, (220 * 1024) / (2 * row_bytes + 1024))));
    const int grid = std::min(rows, sm_count() * per_sm);
    logits_argmax_bulk_kernel<<<grid, kArgmaxThreads, 2 * row_bytes, s>>>(
        logits, V, rows, static_cast<uint32_t>(row_bytes), ids, prob, max_logit,
        calc_prob, device_error_word());
  } else {
    logits_argmax_kernel<<<rows, kArgmaxThreads, 0, s>>>(logits, V, ids, prob,
                                                         max_logit, calc_prob);
  }
  return cudaGetLastError();
}

cudaError_t vocab_merge(const float *part_max, const int *part_id,
                        const float *part_sum, int rows, int tiles, int *ids,
                        float *prob, float *max_logit, int calc_prob,
                        cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  vocab_merge_kernel<<<(rows + 255) / 256, 256, 0, s>>>(
      part_max, part_id, part_sum, rows, tiles, ids, prob, max_logit,
      calc_prob);
  return cudaGetLastError();
}

cudaError_t ctc_collapse(const int *ids, const float *probs, int lines, int T,
                         int blank, int *out_ids, int *out_len,
                         float *out_score, cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  if (T < 0 || !ids || !out_ids || !out_len || !out_score)
    return cudaErrorInvalidValue;
  ctc_collapse_kernel<<<(lines + 255) / 256, 256, 0, s>>>(
      ids, probs, lines, T, blank, out_ids, out_len, out_score);
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
  selected_class_kernel<<<(rows + 7) / 8, 256, 0, s>>>(
      hidden, w, bias, max_logits, out, rows, H, V, class_id);
  return cudaGetLastError();
}

} // namespace pb2
