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

__global__ void __launch_bounds__(256)
    softmax_kernel(const half *__restrict__ x, half *__restrict__ y, int rows,
                   int cols) {
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

// Generic batched matmul, 16x16 output tile per block, fp32 accumulation.
__global__ void __launch_bounds__(256)
    matmul_kernel(const half *__restrict__ a, const half *__restrict__ b,
                  half *__restrict__ y, int m, int n, int k, long long sa,
                  long long sb, long long sy) {
  __shared__ float as[16][17], bs[16][17];
  const int bz = blockIdx.z;
  const half *A = a + bz * sa;
  const half *B = b + bz * sb;
  const int row = blockIdx.y * 16 + threadIdx.y;
  const int col = blockIdx.x * 16 + threadIdx.x;
  float acc = 0.f;
  for (int k0 = 0; k0 < k; k0 += 16) {
    const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
    as[threadIdx.y][threadIdx.x] =
        row < m && ka < k ? __half2float(A[static_cast<long long>(row) * k + ka])
                          : 0.f;
    bs[threadIdx.y][threadIdx.x] =
        kb < k && col < n ? __half2float(B[static_cast<long long>(kb) * n + col])
                          : 0.f;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 16; ++j)
      acc = fmaf(as[threadIdx.y][j], bs[j][threadIdx.x], acc);
    __syncthreads();
  }
  if (row < m && col < n)
    y[bz * sy + static_cast<long long>(row) * n + col] = __float2half_rn(acc);
}

// One block per text line; warp h handles head h (looping if heads > warps).
// Shared memory: the line's qkv rows as fp32 plus one seq x seq score tile
// per warp.
__global__ void __launch_bounds__(256)
    attention_kernel(const half *__restrict__ qkv, half *__restrict__ out,
                     int seq, int heads, int dh, float scale) {
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

// Register-resident form for seq <= 64, head_dim <= 16: one block per text
// line, K and V of every head staged in shared memory as fp32, and each
// thread owning one (head, query row) at a time with its 64 scores, softmax
// and output row in registers. Same rounding points as attention_kernel.
template <int MAXSEQ, int MAXDH>
__global__ void __launch_bounds__(256)
    attention_rows_kernel(const half *__restrict__ qkv, half *__restrict__ out,
                          int seq, int heads, int dh, float scale) {
  extern __shared__ float sm[];
  const int hd = heads * dh;
  const int width = 3 * hd;
  float *ks = sm;                  // [heads][seq][dh]
  float *vs = sm + heads * seq * dh;
  const long long line = blockIdx.x;
  const half *src = qkv + line * seq * width;
  for (int j = threadIdx.x; j < seq * hd; j += blockDim.x) {
    const int i = j / hd, rem = j - i * hd;
    const int h = rem / dh, d = rem - h * dh;
    ks[(h * seq + i) * dh + d] = __half2float(src[i * width + hd + rem]);
    vs[(h * seq + i) * dh + d] = __half2float(src[i * width + 2 * hd + rem]);
  }
  __syncthreads();
  half *dst = out + line * seq * hd;
  for (int task = threadIdx.x; task < heads * seq; task += blockDim.x) {
    const int h = task / seq, i = task - h * seq;
    float q[MAXDH];
#pragma unroll
    for (int d = 0; d < MAXDH; ++d)
      q[d] = d < dh ? round_half(__half2float(src[i * width + h * dh + d]) * scale)
                    : 0.f;
    const float *kh = ks + h * seq * dh;
    float s[MAXSEQ];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < MAXSEQ; ++j) {
      float acc = 0.f;
      if (j < seq) {
#pragma unroll
        for (int d = 0; d < MAXDH; ++d)
          if (d < dh)
            acc = fmaf(q[d], kh[j * dh + d], acc);
        acc = round_half(acc);
        m = fmaxf(m, acc);
      }
      s[j] = acc;
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < MAXSEQ; ++j)
      if (j < seq)
        sum += expf(s[j] - m);
    const float *vh = vs + h * seq * dh;
    float o[MAXDH];
#pragma unroll
    for (int d = 0; d < MAXDH; ++d)
      o[d] = 0.f;
#pragma unroll
    for (int j = 0; j < MAXSEQ; ++j) {
      if (j < seq) {
        const float p = round_half(expf(s[j] - m) / sum);
#pragma unroll
        for (int d = 0; d < MAXDH; ++d)
          if (d < dh)
            o[d] = fmaf(p, vh[j * dh + d], o[d]);
      }
    }
#pragma unroll
    for (int d = 0; d < MAXDH; ++d)
      if (d < dh)
        dst[i * hd + h * dh + d] = __float2half_rn(o[d]);
  }
}

unsigned rows_blocks(int rows) { return static_cast<unsigned>((rows + 7) / 8); }

} // namespace

cudaError_t layernorm(const half *x, const half *scale, const half *bias,
                      half *y, int rows, int cols, float eps, cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  layernorm_kernel<<<rows_blocks(rows), 256, 0, s>>>(x, scale, bias, y, rows,
                                                     cols, eps);
  return cudaGetLastError();
}

cudaError_t softmax_rows(const half *x, half *y, int rows, int cols,
                         cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  softmax_kernel<<<rows_blocks(rows), 256, 0, s>>>(x, y, rows, cols);
  return cudaGetLastError();
}

cudaError_t mean_rows(const half *x, half *y, int rows, int cols,
                      cudaStream_t s) {
  if (rows <= 0)
    return cudaSuccess;
  mean_rows_kernel<<<rows_blocks(rows), 256, 0, s>>>(x, y, rows, cols);
  return cudaGetLastError();
}

cudaError_t mean_nhwc(const half *x, half *y, int batch, int C, int spatial,
                      cudaStream_t s) {
  if (batch <= 0)
    return cudaSuccess;
  mean_nhwc_kernel<<<dim3((C + 31) / 32, batch), 256, 0, s>>>(x, y, C,
                                                               spatial);
  return cudaGetLastError();
}

cudaError_t matmul_batched(const half *a, const half *b, half *y, int batches,
                           int m, int n, int k, long long sa, long long sb,
                           long long sy, cudaStream_t s) {
  if (batches <= 0 || m <= 0 || n <= 0)
    return cudaSuccess;
  dim3 grid((n + 15) / 16, (m + 15) / 16, batches);
  matmul_kernel<<<grid, dim3(16, 16), 0, s>>>(a, b, y, m, n, k, sa, sb, sy);
  return cudaGetLastError();
}

cudaError_t attention(const half *qkv, half *out, int lines, int seq, int heads,
                      int dh, float scale, cudaStream_t s) {
  if (lines <= 0)
    return cudaSuccess;
  if (seq <= 64 && dh <= 16) {
    const size_t kv = sizeof(float) * 2ull * heads * seq * dh;
    if (kv <= 200 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(
          attention_rows_kernel<64, 16>,
          cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kv));
      if (e != cudaSuccess)
        return e;
      attention_rows_kernel<64, 16><<<lines, 256, kv, s>>>(qkv, out, seq, heads,
                                                            dh, scale);
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
  attention_kernel<<<lines, 256, smem, s>>>(qkv, out, seq, heads, dh, scale);
  return cudaGetLastError();
}

} // namespace pb2
