// Sequence-side kernels of the SVTR neck: LayerNorm, row softmax, row mean,
// NHWC global mean, a generic batched matmul and one fused multi-head
// attention kernel per text line.
//
// Reference semantics (ppocrv6-native-server):
//   layernorm  native/src/compiled/runtime.cuh:227-261 (two-pass fp32 mean and
//              variance, rsqrtf(var + eps), affine, fp16 output)
//   softmax    runtime.cuh:189-225 (max, sum expf(x - max), expf/sum)
//   mean       runtime.cuh:189-225, mean_nhwc 290-336
//   matmul     runtime.cuh:1013-1024 (fp16 in/out, fp32 accumulation)
// The reference runs each of these as one 256-thread block per row; here a
// warp owns a row (rows are 40..2048 wide), so a block covers 8 rows.
#include "kernels.h"
#include "ptx.cuh"

namespace pb2 {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void __launch_bounds__(256)
    layernorm_kernel(const half *__restrict__ x, const half *__restrict__ scale,
                     const half *__restrict__ bias, half *__restrict__ y,
                     int rows, int cols, float eps) {
  pdl_begin();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows)
    return;
  const half *xr = x + static_cast<long long>(row) * cols;
  float s = 0.f;
  for (int j = lane; j < cols; j += 32)
    s += __half2float(xr[j]);
  const float mean = warp_sum(s) / cols;
  float v = 0.f;
  for (int j = lane; j < cols; j += 32) {
    const float d = __half2float(xr[j]) - mean;
    v += d * d;
  }
  const float inv = rsqrtf(warp_sum(v) / cols + eps);
  half *yr = y + static_cast<long long>(row) * cols;
  for (int j = lane; j < cols; j += 32)
    yr[j] = __float2half_rn((__half2float(xr[j]) - mean) * inv *
                                __half2float(scale[j]) +
                            __half2float(bias[j]));
}

// Vectorised LayerNorm for cols = 8 * v8 with v8 <= LPR: a row is held in
// registers as 16-byte vectors by a group of LPR lanes (a warp holds 32/LPR
// rows), every warp loading RPW row groups before any arithmetic. Same
// formula as layernorm_kernel (fp32 mean, then the mean of squared
// deviations, y = (x - mean) * rsqrt(var + eps) * scale + bias, one fp16
// rounding); only the order of the fp32 sums differs.
template <int LPR, int RPW>
__global__ void __launch_bounds__(256)
    layernorm_vec_kernel(const half *__restrict__ x, const half *__restrict__ scale,
                         const half *__restrict__ bias, half *__restrict__ y,
                         int rows, int cols, float eps) {
  pdl_begin();
  constexpr int GPW = 32 / LPR; // row groups per warp
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;
  const bool on = l < (cols >> 3);
  const long long row0 = (static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * GPW * RPW;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  uint4 u[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const long long row = row0 + r * GPW + sub;
    u[r] = on && row < rows ? __ldg(reinterpret_cast<const uint4 *>(x + row * cols) + l) : zero;
  }
  const uint4 su = on ? __ldg(reinterpret_cast<const uint4 *>(scale) + l) : zero;
  const uint4 bu = on ? __ldg(reinterpret_cast<const uint4 *>(bias) + l) : zero;
  const half2 *sh = reinterpret_cast<const half2 *>(&su);
  const half2 *bh = reinterpret_cast<const half2 *>(&bu);
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const long long row = row0 + r * GPW + sub;
    const half2 *xh = reinterpret_cast<const half2 *>(&u[r]);
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __half22float2(xh[e]);
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      s += f[e];
#pragma unroll
    for (int o = LPR / 2; o; o >>= 1)
      s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / cols;
    float v = 0.f;
    if (on)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = f[e] - mean;
        v += d * d;
      }
#pragma unroll
    for (int o = LPR / 2; o; o >>= 1)
      v += __shfl_xor_sync(0xffffffffu, v, o);
    const float inv = rsqrtf(v / cols + eps);
    if (on && row < rows) {
      uint4 o;
      half2 *oh = reinterpret_cast<half2 *>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 sc = __half22float2(sh[e]), bi = __half22float2(bh[e]);
        oh[e] = __floats2half2_rn((f[2 * e] - mean) * inv * sc.x + bi.x,
                                  (f[2 * e + 1] - mean) * inv * sc.y + bi.y);
      }
      *(reinterpret_cast<uint4 *>(y + row * cols) + l) = o;
    }
  }
}

__global__ void __launch_bounds__(256)
    softmax_kernel(const half *__restrict__ x, half *__restrict__ y, int rows,
                   int cols) {
  pdl_begin();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows)
    return;
  const half *xr = x + static_cast<long long>(row) * cols;
  float m = -INFINITY;
  for (int j = lane; j < cols; j += 32)
    m = fmaxf(m, __half2float(xr[j]));
  m = warp_max(m);
  float s = 0.f;
  for (int j = lane; j < cols; j += 32)
    s += expf(__half2float(xr[j]) - m);
  s = warp_sum(s);
  half *yr = y + static_cast<long long>(row) * cols;
  for (int j = lane; j < cols; j += 32)
    yr[j] = __float2half_rn(expf(__half2float(xr[j]) - m) / s);
}

__global__ void __launch_bounds__(256)
    mean_rows_kernel(const half *__restrict__ x, half *__restrict__ y, int rows,
                     int cols) {
  pdl_begin();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows)
    return;
  const half *xr = x + static_cast<long long>(row) * cols;
  float s = 0.f;
  for (int j = lane; j < cols; j += 32)
    s += __half2float(xr[j]);
  s = warp_sum(s);
  if (lane == 0)
    y[row] = __float2half_rn(s / cols);
}

// One block per (batch, 32-channel slice); 8 warps stride over the pixels.
__global__ void __launch_bounds__(256)
    mean_nhwc_kernel(const half *__restrict__ x, half *__restrict__ y, int C,
                     int spatial) {
  pdl_begin();
  __shared__ float part[8][33];
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  const int w = threadIdx.x >> 5;
  const long long b = blockIdx.y;
  float s = 0.f;
  if (c < C)
    for (int p = w; p < spatial; p += 8)
      s += __half2float(x[(b * spatial + p) * C + c]);
  part[w][threadIdx.x & 31] = s;
  __syncthreads();
  if (w == 0 && c < C) {
    float t = 0.f;
    for (int j = 0; j < 8; ++j)
      t += part[j][threadIdx.x & 31];
    y[b * C + c] = __float2half_rn(t / spatial);
  }
}

// One block per text line; warp h handles head h (looping if heads > warps).
// Shared memory: the line's qkv rows as fp32 plus one seq x seq score tile
// per warp.
__global__ void __launch_bounds__(256)
    attention_kernel(const half *__restrict__ qkv, half *__restrict__ out,
                     int seq, int heads, int dh, float scale) {
  pdl_begin();
  extern __shared__ float sm[];
  const int width = 3 * heads * dh;
  float *xs = sm;                      // [seq][width]
  float *ss = sm + seq * width;        // [8][seq][seq]
  const long long line = blockIdx.x;
  const half *src = qkv + line * seq * width;
  for (int j = threadIdx.x; j < seq * width; j += blockDim.x)
    xs[j] = __half2float(src[j]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *S = ss + warp * seq * seq;
  for (int h = warp; h < heads; h += 8) {
    const int qo = h * dh, ko = heads * dh + h * dh, vo = 2 * heads * dh + h * dh;
    // S = round(round(q*scale) . k^T)
    for (int e = lane; e < seq * seq; e += 32) {
      const int i = e / seq, j = e - (e / seq) * seq;
      float acc = 0.f;
      for (int d = 0; d < dh; ++d)
        acc = fmaf(round_half(xs[i * width + qo + d] * scale),
                   xs[j * width + ko + d], acc);
      S[e] = round_half(acc);
    }
    __syncwarp();
    // P = round(softmax(S)) row by row
    for (int i = 0; i < seq; ++i) {
      float m = -INFINITY;
      for (int j = lane; j < seq; j += 32)
        m = fmaxf(m, S[i * seq + j]);
      m = warp_max(m);
      float s = 0.f;
      for (int j = lane; j < seq; j += 32)
        s += expf(S[i * seq + j] - m);
      s = warp_sum(s);
      __syncwarp();
      for (int j = lane; j < seq; j += 32)
        S[i * seq + j] = round_half(expf(S[i * seq + j] - m) / s);
      __syncwarp();
    }
    // O = round(P . v)
    half *dst = out + line * seq * heads * dh;
    for (int e = lane; e < seq * dh; e += 32) {
      const int i = e / dh, d = e - (e / dh) * dh;
      float acc = 0.f;
      for (int j = 0; j < seq; ++j)
        acc = fmaf(S[i * seq + j], xs[j * width + vo + d], acc);
      dst[i * heads * dh + h * dh + d] = __float2half_rn(acc);
    }
    __syncwarp();
  }
}

// Staged form: one block per text line. q' = round(q*scale), k, v, the
// scores and the probabilities are all fp16-representable (the reference
// stores each of them as fp16), so they are staged in shared memory as fp16:
// 72 KB per line at 8 heads x 40 tokens, three resident blocks per SM. Rows
// are RS = DP + 8 halves apart so 16-byte reads of consecutive key rows hit
// distinct banks. Three parallel phases: every score (one (head, i, j) per
// thread step), row softmax (one warp per row), every output (one
// (head, i, d) per step). Same rounding points and summation order as
// attention_kernel.
template <int DP>
__global__ void __launch_bounds__(256)
    attention_staged_kernel(const half *__restrict__ qkv,
                            half *__restrict__ out, int seq, int heads, int dh,
                            float scale) {
  pdl_begin();
  constexpr int RS = DP + 8;
  extern __shared__ uint4 att_smem[];
  half *qs = reinterpret_cast<half *>(att_smem); // [heads][seq][RS]
  half *ks = qs + heads * seq * RS;
  half *vs = ks + heads * seq * RS;
  half *ss = vs + heads * seq * RS;               // [heads][seq][seq]
  const int hd = heads * dh;
  const int width = 3 * hd;
  const long long line = blockIdx.x;
  const half *src = qkv + line * seq * width;
  for (int j = threadIdx.x; j < heads * seq * DP; j += blockDim.x) {
    const int d = j % DP, hi = j / DP;
    const int h = hi / seq, i = hi - h * seq;
    half q = __float2half_rn(0.f), k = q, v = q;
    if (d < dh) {
      const half *row = src + i * width + h * dh + d;
      q = __float2half_rn(__half2float(row[0]) * scale);
      k = row[hd];
      v = row[2 * hd];
    }
    qs[hi * RS + d] = q;
    ks[hi * RS + d] = k;
    vs[hi * RS + d] = v;
  }
  __syncthreads();
  // Scores S[h][i][j] = round(q'_i . k_j), d ascending.
  const int nscore = heads * seq * seq;
  for (int e = threadIdx.x; e < nscore; e += blockDim.x) {
    const int j = e % seq, hi = e / seq;
    const int h = hi / seq;
    const uint4 *q8 = reinterpret_cast<const uint4 *>(qs + hi * RS);
    const uint4 *k8 = reinterpret_cast<const uint4 *>(ks + (h * seq + j) * RS);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < DP / 8; ++c) {
      uint4 a = q8[c], b = k8[c];
      const half2 *a2 = reinterpret_cast<const half2 *>(&a);
      const half2 *b2 = reinterpret_cast<const half2 *>(&b);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 x = __half22float2(a2[t]), y = __half22float2(b2[t]);
        acc = fmaf(x.x, y.x, acc);
        acc = fmaf(x.y, y.y, acc);
      }
    }
    ss[e] = __float2half_rn(acc);
  }
  __syncthreads();
  // Row softmax, one warp per (h, i) row: P = round(exp(s - max) / sum).
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int row = warp; row < heads * seq; row += blockDim.x >> 5) {
    half *sr = ss + row * seq;
    float m = -INFINITY;
    for (int j = lane; j < seq; j += 32)
      m = fmaxf(m, __half2float(sr[j]));
    m = warp_max(m);
    float sum = 0.f;
    for (int j = lane; j < seq; j += 32)
      sum += expf(__half2float(sr[j]) - m);
    sum = warp_sum(sum);
    __syncwarp();
    for (int j = lane; j < seq; j += 32)
      sr[j] = __float2half_rn(expf(__half2float(sr[j]) - m) / sum);
  }
  __syncthreads();
  // Outputs O[h][i][d] = round(sum_j P[h][i][j] v[h][j][d]), j ascending.
  half *dst = out + line * seq * hd;
  for (int e = threadIdx.x; e < heads * seq * dh; e += blockDim.x) {
    const int d = e % dh, hi = e / dh;
    const int h = hi / seq, i = hi - h * seq;
    const half *pr = ss + hi * seq;
    const half *vc = vs + h * seq * RS + d;
    float acc = 0.f;
    for (int j = 0; j < seq; ++j)
      acc = fmaf(__half2float(pr[j]), __half2float(vc[j * RS]), acc);
    dst[i * hd + h * dh + d] = __float2half_rn(acc);
  }
}

// Fixed-length attention (seq == SEQ, head_dim <= 16), one line per block,
// one thread per (head, query) row: the same arithmetic as
// attention_rows_kernel below (q' = round(q*scale); S = round(q'.k) with the
// even and odd dimensions summed in two fp32 chains; P = round(exp(S - max)
// * (1/sum)); O = round(sum_j P_j v_j), j ascending), with q', K and V
// staged once in shared memory as fp32 ([head][pos][16], zero-padded) so
// every multiply-add pair is one packed fp32 FMA (fma.rn.f32x2 rounds each
// lane like fmaf: bit-identical results) fed by 16-byte shared loads, and
// the score row a fixed-size register array. The line's rows are read with
// 16-byte loads when the row width allows.
template <int SEQ>
__global__ void __launch_bounds__(512)
    attention_f32_kernel(const half *__restrict__ qkv, half *__restrict__ out,
                         int heads, int dh, float scale, FastDiv by_dh, int vec) {
  pdl_begin();
  constexpr int DP = 16;
  extern __shared__ float4 att32_smem[];
  float *qs = reinterpret_cast<float *>(att32_smem); // [heads][SEQ][DP]
  float *ks = qs + heads * SEQ * DP;
  float *vs = ks + heads * SEQ * DP;
  const int hd = heads * dh;
  const int width = 3 * hd;
  const long long line = blockIdx.x;
  const half *src = qkv + line * SEQ * width;
  const int tid = threadIdx.x;
  // Padding dimensions d in [dh, 16) of q', K and V are zero.
  for (int e = tid; e < 3 * heads * SEQ * (DP - dh); e += blockDim.x) {
    const int r = e / (DP - dh);
    qs[r * DP + dh + (e - r * (DP - dh))] = 0.f;
  }
  auto put = [&](int c, int j, float v) {
    const int sec = c >= 2 * hd ? 2 : c >= hd ? 1 : 0;
    const uint32_t cc = static_cast<uint32_t>(c - sec * hd);
    const uint32_t h = by_dh.div(cc), d = cc - h * dh;
    if (sec == 0)
      v = round_half(v * scale);
    qs[sec * heads * SEQ * DP + (h * SEQ + j) * DP + d] = v;
  };
  if (vec) {
    // width is a multiple of 8: whole 16-byte groups of one row
    const int groups = width >> 3;
    for (int e = tid; e < SEQ * groups; e += blockDim.x) {
      const int j = e / groups, c8 = (e - j * groups) * 8;
      const uint4 u = __ldg(reinterpret_cast<const uint4 *>(src + j * width + c8));
      const half2 *h2 = reinterpret_cast<const half2 *>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h2[i]);
        put(c8 + 2 * i, j, f.x);
        put(c8 + 2 * i + 1, j, f.y);
      }
    }
  } else {
    for (int e = tid; e < SEQ * width; e += blockDim.x) {
      const int j = e / width;
      put(e - j * width, j, __half2float(src[e]));
    }
  }
  __syncthreads();
  const int row = tid;
  if (row >= heads * SEQ)
    return;
  const int h = row / SEQ, i = row - h * SEQ;
  const float4 *q4 = reinterpret_cast<const float4 *>(qs + row * DP);
  float2 q[8];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float4 v = q4[t];
    q[2 * t] = make_float2(v.x, v.y);
    q[2 * t + 1] = make_float2(v.z, v.w);
  }
  const float4 *k4 = reinterpret_cast<const float4 *>(ks + h * SEQ * DP);
  float sc[SEQ];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < SEQ; ++j) {
    float2 e = make_float2(0.f, 0.f);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float4 kv = k4[j * 4 + t];
      ffma2(e, q[2 * t], make_float2(kv.x, kv.y));
      ffma2(e, q[2 * t + 1], make_float2(kv.z, kv.w));
    }
    sc[j] = round_half(e.x + e.y);
    m = fmaxf(m, sc[j]);
  }
  const float mL = m * kLog2e;
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < SEQ; ++j) {
    sc[j] = ex2_ftz(fmaf(sc[j], kLog2e, -mL));
    sum += sc[j];
  }
  const float inv = 1.f / sum;
  float2 o[8];
#pragma unroll
  for (int t = 0; t < 8; ++t)
    o[t] = make_float2(0.f, 0.f);
  const float4 *v4 = reinterpret_cast<const float4 *>(vs + h * SEQ * DP);
#pragma unroll
  for (int j = 0; j < SEQ; ++j) {
    const float p = round_half(sc[j] * inv);
    const float2 pp = make_float2(p, p);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float4 vv = v4[j * 4 + t];
      ffma2(o[2 * t], pp, make_float2(vv.x, vv.y));
      ffma2(o[2 * t + 1], pp, make_float2(vv.z, vv.w));
    }
  }
  half *dst = out + (line * SEQ + i) * hd + h * dh;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    if (2 * t < dh)
      dst[2 * t] = __float2half_rn(o[t].x);
    if (2 * t + 1 < dh)
      dst[2 * t + 1] = __float2half_rn(o[t].y);
  }
}

// Short-sequence attention (seq <= SMAX, head_dim <= 16), one line per
// block, one thread per (head, query) row doing the whole row: the line's
// q' = round(q*scale), K and V are staged in shared memory ([head][pos][16],
// zero-padded) with 16-byte loads where the row layout allows; the thread
// keeps its q' and its row of scores in registers, S = round(q'.k) (fp16
// operands, fp32 sums, two interleaved chains over d), P = round(exp(S -
// max) * (1/sum)) with exp on the special-function unit, O = round(sum_j
// P_j v_j) (j ascending, fp32). The K/V reads are warp-wide broadcasts (a
// warp's rows share a head); every multiply-add is one mixed-precision
// instruction.
template <int SMAX>
__global__ void __launch_bounds__(512)
    attention_rows_kernel(const half *__restrict__ qkv, half *__restrict__ out,
                          int seq, int heads, int dh, float scale,
                          FastDiv by_hd, FastDiv by_dh, FastDiv by_seq, int vec) {
  pdl_begin();
  constexpr int DP = 16;
  extern __shared__ uint4 att_smem[];
  half *qs = reinterpret_cast<half *>(att_smem); // [heads][seq][DP]
  half *ks = qs + heads * seq * DP;
  half *vs = ks + heads * seq * DP;
  const int hd = heads * dh;
  const int width = 3 * hd;
  const long long line = blockIdx.x;
  const half *src = qkv + line * seq * width;
  const half zero = __float2half_rn(0.f);
  if (dh < DP)
    for (int e = threadIdx.x; e < heads * seq * DP; e += blockDim.x)
      qs[e] = ks[e] = vs[e] = zero;
  __syncthreads();
  auto put = [&](uint32_t c, int j, half q, half k, half v) {
    const uint32_t h = by_dh.div(c), d = c - h * dh;
    const int at = (h * seq + j) * DP + d;
    qs[at] = __float2half_rn(__half2float(q) * scale);
    ks[at] = k;
    vs[at] = v;
  };
  if (vec) {
    // hd and the row width are multiples of 8 halves: whole 16-byte groups
    const int groups = hd >> 3;
    for (int e = threadIdx.x; e < seq * groups; e += blockDim.x) {
      const int j = e / groups, c8 = (e - j * groups) * 8;
      const uint4 *row = reinterpret_cast<const uint4 *>(src + j * width + c8);
      const uint4 uq = row[0], uk = row[hd >> 3], uv = row[hd >> 2];
      const half *hq = reinterpret_cast<const half *>(&uq);
      const half *hk = reinterpret_cast<const half *>(&uk);
      const half *hv = reinterpret_cast<const half *>(&uv);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        put(c8 + i, j, hq[i], hk[i], hv[i]);
    }
  } else {
    for (uint32_t e = threadIdx.x; e < static_cast<uint32_t>(seq * hd); e += blockDim.x) {
      const uint32_t j = by_hd.div(e), c = e - j * hd;
      put(c, j, src[j * width + c], src[j * width + hd + c], src[j * width + 2 * hd + c]);
    }
  }
  __syncthreads();
  const int rows = heads * seq;
  for (int row = threadIdx.x; row < rows; row += blockDim.x) {
    const int h = static_cast<int>(by_seq.div(row));
    const int i = row - h * seq;
    const uint4 *q4 = reinterpret_cast<const uint4 *>(qs + row * DP);
    const uint4 qa = q4[0], qb = q4[1];
    const uint32_t q[DP / 2] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    const uint4 *k4 = reinterpret_cast<const uint4 *>(ks + h * seq * DP);
    float sc[SMAX];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < SMAX; ++j) {
      if (j < seq) {
        const uint4 a = k4[2 * j], b = k4[2 * j + 1];
        float e0 = 0.f, e1 = 0.f;
        fma2_h(e0, e1, q[0], a.x);
        fma2_h(e0, e1, q[1], a.y);
        fma2_h(e0, e1, q[2], a.z);
        fma2_h(e0, e1, q[3], a.w);
        fma2_h(e0, e1, q[4], b.x);
        fma2_h(e0, e1, q[5], b.y);
        fma2_h(e0, e1, q[6], b.z);
        fma2_h(e0, e1, q[7], b.w);
        sc[j] = round_half(e0 + e1);
        m = fmaxf(m, sc[j]);
      }
    }
    const float mL = m * kLog2e;
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < SMAX; ++j)
      if (j < seq) {
        sc[j] = ex2_ftz(fmaf(sc[j], kLog2e, -mL));
        sum += sc[j];
      }
    const float inv = 1.f / sum;
    float o[DP];
#pragma unroll
    for (int d = 0; d < DP; ++d)
      o[d] = 0.f;
    const uint4 *v4 = reinterpret_cast<const uint4 *>(vs + h * seq * DP);
#pragma unroll
    for (int j = 0; j < SMAX; ++j) {
      if (j < seq) {
        const uint32_t pb = __half_as_ushort(__float2half_rn(sc[j] * inv));
        const uint32_t pp = pb | (pb << 16);
        const uint4 a = v4[2 * j], b = v4[2 * j + 1];
        fma2_h(o[0], o[1], pp, a.x);
        fma2_h(o[2], o[3], pp, a.y);
        fma2_h(o[4], o[5], pp, a.z);
        fma2_h(o[6], o[7], pp, a.w);
        fma2_h(o[8], o[9], pp, b.x);
        fma2_h(o[10], o[11], pp, b.y);
        fma2_h(o[12], o[13], pp, b.z);
        fma2_h(o[14], o[15], pp, b.w);
      }
    }
    half *dst = out + (line * seq + i) * hd + h * dh;
#pragma unroll
    for (int d = 0; d < DP; ++d)
      if (d < dh)
        dst[d] = __float2half_rn(o[d]);
  }
}

unsigned rows_blocks(int rows) { return static_cast<unsigned>((rows + 7) / 8); }

} // namespace

cudaError_t layernorm(const half *x, const half *scale, const half *bias,
                      half *y, int rows, int cols, float eps, cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  const bool vec = cols % 8 == 0 && cols > 32 && cols <= 256 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                     reinterpret_cast<uintptr_t>(scale) | reinterpret_cast<uintptr_t>(bias)) & 15) == 0;
  if (vec) {
    constexpr int RPW = 4;
    auto launch = [&](auto kernel, int lpr) {
      const long long per_block = 8LL * (32 / lpr) * RPW;
      launch_pdl(kernel, static_cast<unsigned>((rows + per_block - 1) / per_block), 256, 0, s, x,
          scale, bias, y, rows, cols, eps);
      return cudaGetLastError();
    };
    if (cols <= 64)
      return launch(layernorm_vec_kernel<8, RPW>, 8);
    if (cols <= 128)
      return launch(layernorm_vec_kernel<16, RPW>, 16);
    return launch(layernorm_vec_kernel<32, RPW>, 32);
  }
  launch_pdl(layernorm_kernel, rows_blocks(rows), 256, 0, s, x, scale, bias, y, rows, cols, eps);
  return cudaGetLastError();
}

cudaError_t softmax_rows(const half *x, half *y, int rows, int cols,
                         cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  launch_pdl(softmax_kernel, rows_blocks(rows), 256, 0, s, x, y, rows, cols);
  return cudaGetLastError();
}

cudaError_t mean_rows(const half *x, half *y, int rows, int cols,
                      cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  launch_pdl(mean_rows_kernel, rows_blocks(rows), 256, 0, s, x, y, rows, cols);
  return cudaGetLastError();
}

cudaError_t mean_nhwc(const half *x, half *y, int batch, int C, int spatial,
                      cudaStream_t s) {
  if (batch <= 0)
    return cudaSuccess;
  launch_pdl(mean_nhwc_kernel, dim3((C + 31) / 32, batch), 256, 0, s, x, y, C, spatial);
  return cudaGetLastError();
}

cudaError_t matmul_batched(const half *a, const half *b, half *y, int batches,
                           int m, int n, int k, long long sa, long long sb,
                           long long sy, cudaStream_t s) {
  if (batches <= 0 || m <= 0 || n <= 0)
    return cudaSuccess;
  if (k < 0)
    return cudaErrorInvalidValue;
  // Tensor cores (matmul_tc.cu), one launch per 65535 batches (the grid's z
  // limit). With k = 0 the operands may be null and are not offset.
  for (long long b0 = 0; b0 < batches; b0 += 65535) {
    const int nb = static_cast<int>(batches - b0 < 65535 ? batches - b0 : 65535);
    const cudaError_t e = matmul_tc(k > 0 ? a + b0 * sa : a, k > 0 ? b + b0 * sb : b, y + b0 * sy, nb, m, n, k,
                                    sa, sb, sy, s);
    if (e != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

cudaError_t attention(const half *qkv, half *out, int lines, int seq, int heads,
                      int dh, float scale, cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  if (attention_tc_supported(seq, dh) && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(out) & 3) == 0 &&
      static_cast<long long>(lines) * seq * 3 * heads * dh < (1ll << 31))
    return attention_tc(qkv, out, lines, seq, heads, dh, scale, s);
  return attention_simt(qkv, out, lines, seq, heads, dh, scale, s);
}

cudaError_t attention_simt(const half *qkv, half *out, int lines, int seq, int heads,
                           int dh, float scale, cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  if (dh <= 16 && seq == 40 && heads * 40 <= 512) {
    const int threads = (heads * 40 + 31) / 32 * 32;
    const size_t smem = sizeof(float) * 3ull * heads * 40 * 16;
    const int vec = (3 * heads * dh) % 8 == 0 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0;
    if (smem <= 200 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(attention_f32_kernel<40>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess)
        return e;
      launch_pdl(attention_f32_kernel<40>, lines, threads, smem, s, qkv, out, heads, dh, scale,
          FastDiv(dh), vec);
      return cudaGetLastError();
    }
  }
  if (dh <= 16 && seq <= 64) {
    const int rows = heads * seq;
    const int threads = rows >= 512 ? 512 : (rows + 31) / 32 * 32;
    const size_t smem = sizeof(half) * 3ull * heads * seq * 16;
    const int vec = (heads * dh) % 8 == 0 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0;
    if (smem <= 48 * 1024) {
      launch_pdl(attention_rows_kernel<64>, lines, threads, smem, s, qkv, out, seq, heads, dh,
          scale, FastDiv(heads * dh), FastDiv(dh), FastDiv(seq), vec);
      return cudaGetLastError();
    }
  }
  if (dh <= 32) {
    const int dp = dh <= 16 ? 16 : 32;
    const size_t staged =
        sizeof(half) * (3ull * heads * seq * (dp + 8) + 1ull * heads * seq * seq);
    if (staged <= 200 * 1024) {
      auto kernel = dp == 16 ? attention_staged_kernel<16>
                             : attention_staged_kernel<32>;
      cudaError_t e = cudaFuncSetAttribute(
          kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
          static_cast<int>(staged));
      if (e != cudaSuccess)
        return e;
      launch_pdl(kernel, lines, 256, staged, s, qkv, out, seq, heads, dh, scale);
      return cudaGetLastError();
    }
  }
  const size_t smem =
      sizeof(float) * (static_cast<size_t>(seq) * 3 * heads * dh +
                       8ull * seq * seq);
  if (smem > 200 * 1024)
    return cudaErrorInvalidValue;
  // Per-device function attribute; cheap, so set on every call.
  cudaError_t e = cudaFuncSetAttribute(
      attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
      static_cast<int>(smem));
  if (e != cudaSuccess)
    return e;
  launch_pdl(attention_kernel, lines, 256, smem, s, qkv, out, seq, heads, dh, scale);
  return cudaGetLastError();
}

} // namespace pb2
