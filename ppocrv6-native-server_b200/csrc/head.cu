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

struct Best {
  float m;
  int id;
  float s;
};

__device__ __forceinline__ Best merge(Best a, Best b) {
  // (max, lowest id) plus rescaled exp-sums.
  Best r;
  const bool take_b = b.m > a.m || (b.m == a.m && b.id < a.id);
  r.m = take_b ? b.m : a.m;
  r.id = take_b ? b.id : a.id;
  const float sa = a.s == 0.f ? 0.f : a.s * __expf(a.m - r.m);
  const float sb = b.s == 0.f ? 0.f : b.s * __expf(b.m - r.m);
  r.s = sa + sb;
  return r;
}

// One 256-thread block per row of fp16 logits.
__global__ void __launch_bounds__(256)
    logits_argmax_kernel(const half *__restrict__ logits, int V,
                         int *__restrict__ ids, float *__restrict__ prob,
                         float *__restrict__ max_logit, int calc_prob) {
  __shared__ Best red[8];
  const long long row = blockIdx.x;
  const half *lr = logits + row * V;
  Best b{-FLT_MAX, INT_MAX, 0.f};
  for (int j = threadIdx.x; j < V; j += 256) {
    const float l = __half2float(lr[j]);
    if (l > b.m) {
      b.s = (b.s == 0.f ? 0.f : b.s * __expf(b.m - l)) + 1.f;
      b.m = l;
      b.id = j;
    } else {
      b.s += __expf(l - b.m);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    Best other;
    other.m = __shfl_xor_sync(0xffffffffu, b.m, o);
    other.id = __shfl_xor_sync(0xffffffffu, b.id, o);
    other.s = __shfl_xor_sync(0xffffffffu, b.s, o);
    b = merge(b, other);
  }
  if ((threadIdx.x & 31) == 0)
    red[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    Best t = red[0];
    for (int w = 1; w < 8; ++w)
      t = merge(t, red[w]);
    ids[row] = t.id;
    max_logit[row] = t.m;
    prob[row] = calc_prob ? 1.f / t.s : 1.f;
  }
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

} // namespace

cudaError_t logits_argmax_prob(const half *logits, int rows, int V, int *ids,
                               float *prob, float *max_logit, int calc_prob,
                               cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  if (V <= 0 || !ids || !prob || !max_logit)
    return cudaErrorInvalidValue;
  logits_argmax_kernel<<<rows, 256, 0, s>>>(logits, V, ids, prob, max_logit,
                                            calc_prob);
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
