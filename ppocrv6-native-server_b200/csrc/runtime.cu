// Operator API implementation: every method validates its operator form at
// build time and appends a closure that launches the matching sm_100a kernel.
// Dispatch mirrors the reference's Runtime (native/src/compiled/runtime.cuh)
// method by method; the kernels behind it are the ones in kernels.h.
#include "kernels.h"
#include "runtime.h"

using namespace pb2;

namespace {

void check(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

std::string shape_str(const Shape &s) {
  std::string r = "{";
  for (size_t i = 0; i < s.size(); ++i)
    r += (i ? "," : "") + std::to_string(s[i]);
  return r + "}";
}

// Right-aligned numpy broadcasting of `source` into `dest` (rank <= 6), as
// the reference's indexer() (runtime.cuh:47-62).
Gather broadcast_map(const Shape &source, const Shape &dest) {
  if (dest.size() > 6 || source.size() > dest.size())
    throw std::runtime_error("unsupported broadcast rank");
  Gather g;
  g.rank = static_cast<int>(dest.size());
  long long stride = 1;
  for (int j = g.rank - 1; j >= 0; --j) {
    g.shape[j] = dest[j];
    const int k = j - static_cast<int>(dest.size() - source.size());
    if (k >= 0) {
      g.stride[j] = source[k] == 1 ? 0 : stride;
      stride *= source[k];
    }
  }
  return g;
}

} // namespace

Runtime::Runtime() {
  CU(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
}

Runtime::~Runtime() {
  if (stream)
    cudaStreamSynchronize(stream);
  ops.clear();
  prepare.clear();
  for (void *p : owned_)
    cudaFree(p);
  if (stream)
    cudaStreamDestroy(stream);
}

void *Runtime::own(size_t bytes) {
  void *p = nullptr;
  CU(cudaMalloc(&p, bytes));
  owned_.push_back(p);
  return p;
}

// A fused pair reads the first op's inputs and writes the second op's
// output in one kernel; the arena planner may have given that output the
// space of a first-op input that dies after the first op, so fusion
// requires the two ranges to be disjoint.
static bool disjoint(const Scalar *a, size_t na, const Scalar *b, size_t nb) {
  return a + na <= b || b + nb <= a;
}

bool Runtime::is_constant(const Scalar *p, size_t elements) const {
  return weights && weight_elements && p >= weights &&
         p + elements <= weights + weight_elements;
}

void Runtime::add(const char *name, std::function<void()> f) {
  op_names.resize(ops.size());
  op_names.emplace_back(name);
  ops.push_back(std::move(f));
  last_dw_.op = -1;
  last_dc_.op = -1;
  last_gemm_.op = -1;
}

void Runtime::reads(std::initializer_list<int> ids) {
  for (size_t i = 0; i < fused_.size();) {
    bool hit = false;
    for (int id : ids)
      hit |= id >= 0 && id == fused_[i].virt;
    if (!hit) {
      ++i;
      continue;
    }
    // Split: the first op (writing the intermediate) then the second, in
    // the pair's two slots (the second held an empty placeholder).
    const FusedDw f = fused_[i];
    fused_.erase(fused_.begin() + static_cast<long>(i));
    op_names.resize(ops.size());
    ops[f.op] = f.dw_op;
    op_names[f.op] = f.first_name;
    ops[f.op + 1] = f.pw_op;
    op_names[f.op + 1] = f.second_name;
  }
}

void Runtime::add_fused_placeholder() {
  // Keeps one op slot per graph operator: the fused pair's second slot
  // launches nothing (and is reported as "fused") unless the pair splits.
  add("fused", [] {});
}

namespace pb2 {
// Kernel choice for an NHWC convolution (shared by Runtime::conv and the
// extern "C" entry point): depthwise -> SIMT depthwise; 1x1 stride 1 ->
// tcgen05 GEMM; other stride-1 -> tcgen05 implicit GEMM; small-Ci strided
// (the stem) -> SIMT direct conv. Returns cudaErrorNotSupported otherwise.
cudaError_t conv_nhwc(const half *x, const half *w, const half *bias, half *y,
                      int B, int C, int H, int W, int Co, int KH, int KW,
                      int SH, int SW, int PH, int PW, int groups, int act,
                      cudaStream_t stream) {
  const int OH = (H + 2 * PH - KH) / SH + 1, OW = (W + 2 * PW - KW) / SW + 1;
  if (groups == C && Co == C) {
    if (C % 8)
      return cudaErrorNotSupported;
    return depthwise(x, w, bias, y, B, C, H, W, OH, OW, KH, KW, SH, SW, PH, PW,
                     act, stream);
  }
  if (groups != 1)
    return cudaErrorNotSupported;
  GemmEpilogue e;
  e.bias = bias;
  e.out = y;
  e.ldo = Co;
  e.act = act;
  if (KH == 1 && KW == 1 && SH == 1 && SW == 1 && PH == 0 && PW == 0 &&
      C % 8 == 0 && Co % 8 == 0)
    return tc_gemm(x, B * H * W, C, C, w, Co, C, e, stream);
  if (SH == 1 && SW == 1 && C % 8 == 0 && Co % 8 == 0) {
    ConvShape s{B, H, W, C, Co, KH, KW, PH, PW};
    return tc_conv(x, w, s, e, stream);
  }
  if (Co % 8 == 0 && static_cast<size_t>(Co) * KH * KW * C * 4 <= 48 * 1024)
    return direct_conv(x, w, bias, y, B, C, H, W, Co, OH, OW, KH, KW, SH, SW,
                       PH, PW, act, stream);
  return cudaErrorNotSupported;
}
} // namespace pb2

void Runtime::conv(int ai, int wi, int yi, Shape xs, Shape ws, Shape ys,
                   Shape pad, Shape stride, Shape dilation, int groups,
                   bool channels_last, bool input_channels_last, int bias_id,
                   int activation) {
  if (xs.size() != 4 || ws.size() != 4 || ys.size() != 4 || pad.size() != 2 ||
      stride.size() != 2 || dilation.size() != 2)
    throw std::runtime_error("conv expects rank-4 shapes");
  if (!channels_last || !input_channels_last)
    throw std::runtime_error("B200 conv supports channels-last tensors only");
  if (dilation != Shape{1, 1})
    throw std::runtime_error("B200 conv supports dilation 1 only");
  const int B = xs[0], C = xs[1], H = xs[2], W = xs[3];
  const int Co = ys[1], OH = ys[2], OW = ys[3], KH = ws[2], KW = ws[3];
  if ((H + 2 * pad[0] - KH) / stride[0] + 1 != OH ||
      (W + 2 * pad[1] - KW) / stride[1] + 1 != OW)
    throw std::runtime_error("conv output shape mismatch: " + shape_str(xs) +
                             " -> " + shape_str(ys));
  const bool dw = groups == C && ws[0] == C && ws[1] == 1 && Co == C;
  const char *name = nullptr;
  if (dw)
    name = C % 8 == 0 ? "depthwise" : nullptr;
  else if (groups == 1 && ws[1] == C && ws[0] == Co) {
    if (KH == 1 && KW == 1 && stride == Shape{1, 1} && pad == Shape{0, 0} &&
        C % 8 == 0 && Co % 8 == 0)
      name = "gemm1x1";
    else if (stride == Shape{1, 1} && C % 8 == 0 && Co % 8 == 0)
      name = "implicit_conv";
    else if (Co % 8 == 0 &&
             static_cast<size_t>(Co) * KH * KW * C * 4 <= 48 * 1024)
      name = "direct_conv";
  }
  if (!name)
    throw std::runtime_error("unsupported conv form " + shape_str(xs) + " w=" +
                             shape_str(ws) + " groups=" +
                             std::to_string(groups) + " stride=" +
                             shape_str(stride));
  reads({ai, wi, bias_id});
  add(name, [=] {
    check(conv_nhwc(t[ai], t[wi], bias_id >= 0 ? t[bias_id] : nullptr, t[yi],
                    B, C, H, W, Co, KH, KW, stride[0], stride[1], pad[0],
                    pad[1], groups, activation, stream),
          name);
  });
  // A same-size depthwise conv may open a fused depthwise + pointwise block
  // with the gemm_epilogue that follows it.
  if (dw && KH == KW && stride == Shape{1, 1} && pad == Shape{KH / 2, KW / 2} &&
      dwpw_supported(C, KH, 64))
    last_dw_ = {static_cast<int>(ops.size()) - 1, ai, wi, yi, bias_id, activation, B, C, H, W, KH};
}

void Runtime::deconv(int ai, int wi, int yi, Shape xs, Shape ws, Shape ys,
                     Shape pad, Shape stride, Shape dilation,
                     bool channels_last, int bias_id, int activation) {
  reads({ai, wi, bias_id});
  // ONNX ConvTranspose weight [Ci][Co][KH][KW], stored [Ci][KH][KW][Co] after
  // the channels-last pass.
  if (!channels_last || pad != Shape{0, 0} || dilation != Shape{1, 1} ||
      stride[0] != ws[2] || stride[1] != ws[3])
    throw std::runtime_error("deconv supports channels-last, kernel == stride, "
                             "no padding only");
  const int B = xs[0], Ci = xs[1], H = xs[2], W = xs[3], Co = ws[1];
  const int KH = ws[2], KW = ws[3];
  if (ys[1] != Co || ys[2] != H * KH || ys[3] != W * KW)
    throw std::runtime_error("deconv output shape mismatch");
  const size_t wn = static_cast<size_t>(Ci) * KH * KW * Co;
  if (Co % 64 == 0 && Ci % 8 == 0 && is_constant(t[wi], wn) &&
      (bias_id < 0 || is_constant(t[bias_id], static_cast<size_t>(Co)))) {
    // Tensor-core path: the filter re-laid K-major per tap and the bias
    // repeated per tap, once, at prepare time.
    half *wp = static_cast<half *>(own(wn * sizeof(half)));
    half *bp = bias_id >= 0 ? static_cast<half *>(own(sizeof(half) * KH * KW * Co)) : nullptr;
    prepare.emplace_back([=] {
      check(deconv_pack(t[wi], bias_id >= 0 ? t[bias_id] : nullptr, wp, bp, Ci,
                        Co, KH, KW, stream),
            "pack deconv weight");
    });
    add("deconv_tc", [=] {
      check(tc_deconv(t[ai], wp, bp, t[yi], B, H, W, Ci, Co, KH, KW, activation,
                      stream),
            "tc_deconv");
    });
    if (Co == 64 && KH == 2 && KW == 2)
      last_dc_ = {static_cast<int>(ops.size()) - 1, ai, yi, B, H, W, Ci, Co, KH, KW, activation, wp, bp};
    return;
  }
  auto plain = [=] {
    check(deconv_kxk(t[ai], t[wi], bias_id >= 0 ? t[bias_id] : nullptr, t[yi],
                     B, H, W, Ci, Co, KH, KW, activation, stream),
          "deconv");
  };
  const PendingDeconv d = last_dc_;
  if (d.op >= 0 && d.op == static_cast<int>(ops.size()) - 1 && ai == d.yi && wi != d.yi &&
      bias_id != d.yi && Ci == 64 && Co == 1 && KH == 2 && KW == 2 && B == d.B &&
      H == 2 * d.H && W == 2 * d.W && is_constant(t[wi], wn) &&
      (bias_id < 0 || is_constant(t[bias_id], 1)) &&
      disjoint(t[d.ai], static_cast<size_t>(d.B) * d.H * d.W * d.Ci, t[yi],
               static_cast<size_t>(B) * 4 * H * W)) {
    // DB tail: the 64 -> 1 conv reduces the previous transposed conv's
    // outputs inside its epilogue; the 64-channel map is not materialised.
    reads({wi, bias_id});
    float *w2 = static_cast<float *>(own(wn * sizeof(float)));
    prepare.emplace_back([=] { check(widen_f16(t[wi], w2, static_cast<int>(wn), stream), "widen tail filter"); });
    fused_.push_back({d.op, d.yi, ops[d.op], plain, "deconv_tc", "deconv"});
    ops[d.op] = [=] {
      check(tc_deconv_db_tail(t[d.ai], d.wp, d.bp, d.act, w2, bias_id >= 0 ? t[bias_id] : nullptr, activation,
                              t[yi], d.B, d.H, d.W, d.Ci, stream),
            "tc_deconv_db_tail");
    };
    op_names.resize(ops.size());
    op_names[d.op] = "deconv_db_tail";
    add_fused_placeholder();
    return;
  }
  add("deconv", plain);
}

void Runtime::gemm_epilogue(int ai, int wi, int bi, int ri, int yi, int rows,
                            int ci, int co, int activation) {
  if (ci % 8 || co % 8)
    throw std::runtime_error("gemm_epilogue needs ci, co multiples of 8");
  auto pw = [=] {
    GemmEpilogue e;
    e.bias = bi >= 0 ? t[bi] : nullptr;
    e.residual = ri >= 0 ? t[ri] : nullptr;
    e.ldr = co;
    e.out = t[yi];
    e.ldo = co;
    e.act = activation;
    check(tc_gemm(t[ai], rows, ci, ci, t[wi], co, ci, e, stream), "tc_gemm");
  };
  const PendingDw d = last_dw_;
  if (d.op >= 0 && d.op == static_cast<int>(ops.size()) - 1 && ai == d.yi && ri < 0 && wi != d.yi &&
      bi != d.yi && rows == d.B * d.H * d.W && ci == d.C && dwpw_supported(d.C, d.K, co) &&
      disjoint(t[d.ai], static_cast<size_t>(rows) * ci, t[yi], static_cast<size_t>(rows) * co)) {
    // Fused depthwise + pointwise block: the depthwise output stays on chip.
    reads({wi, bi});
    fused_.push_back({d.op, d.yi, ops[d.op], pw});
    ops[d.op] = [=] {
      check(dwpw_block(t[d.ai], t[d.wi], d.bias_id >= 0 ? t[d.bias_id] : nullptr, d.act, t[wi],
                       bi >= 0 ? t[bi] : nullptr, activation, t[yi], d.B, d.H, d.W, d.C, d.K, co, stream),
            "dwpw_block");
    };
    op_names.resize(ops.size());
    op_names[d.op] = "dwpw_block";
    add_fused_placeholder();
    return;
  }
  reads({ai, wi, bi, ri});
  add("gemm_epilogue", pw);
  if (ri < 0)
    last_gemm_ = {static_cast<int>(ops.size()) - 1, ai, wi, bi, yi, rows, ci, co, activation};
}

void Runtime::matmul(int a, int b, int y, int batches, int m, int n, int k) {
  reads({a, b});
  // Constant right-hand side (a linear layer): re-lay [k][n] as K-major
  // [n][k] once, then run it on the tensor-core GEMM.
  if (batches == 1 && k % 8 == 0 && n % 8 == 0 && t[b] &&
      is_constant(t[b], static_cast<size_t>(k) * n)) {
    half *packed = static_cast<half *>(own(static_cast<size_t>(k) * n * 2));
    prepare.emplace_back([=] {
      check(transpose2d(t[b], packed, 1, k, n, stream), "pack matmul weight");
    });
    add("matmul_const", [=] {
      GemmEpilogue e;
      e.out = t[y];
      e.ldo = n;
      // The reference's matmul has no fused epilogue: output = round(acc).
      check(tc_gemm(t[a], m, k, k, packed, n, k, e, stream), "tc_gemm");
    });
    return;
  }
  add("matmul", [=] {
    check(matmul_batched(t[a], t[b], t[y], batches, m, n, k,
                         static_cast<long long>(m) * k,
                         static_cast<long long>(k) * n,
                         static_cast<long long>(m) * n, stream),
          "matmul");
  });
}

void Runtime::layernorm(int a, int scale, int bias, int y, int rows, int cols,
                        float epsilon) {
  reads({a, scale, bias});
  add("layernorm", [=] {
    check(::pb2::layernorm(t[a], t[scale], t[bias], t[y], rows, cols, epsilon,
                           stream),
          "layernorm");
  });
}

void Runtime::softmax(int a, int y, int rows, int cols) {
  reads({a});
  add("softmax", [=] {
    check(softmax_rows(t[a], t[y], rows, cols, stream), "softmax");
  });
}

void Runtime::binary(int a, int b, int y, Shape as, Shape bs, Shape ys,
                     int op) {
  reads({a, b});
  const Gather ga = broadcast_map(as, ys), gb = broadcast_map(bs, ys);
  const long long n = count(ys);
  add("binary", [=] {
    check(::pb2::binary(t[a], t[b], t[y], n, ga, gb, op, stream), "binary");
  });
}

void Runtime::binary_flat_op(int a, int b, int y, int n, int ad, int am,
                             int bd, int bm, int op) {
  reads({a, b});
  add("binary_fast", [=] {
    check(binary_flat(t[a], t[b], t[y], n, ad, am, bd, bm, op, stream),
          "binary_fast");
  });
}

void Runtime::unary(int a, int y, int n, int op, float alpha, float beta) {
  reads({a});
  add("unary", [=] {
    check(::pb2::unary(t[a], t[y], n, op, alpha, beta, stream), "unary");
  });
}

void Runtime::transpose(int a, int y, Shape xs, Shape ys, Shape perm) {
  reads({a});
  int batch = 0, rows = 0, cols = 0;
  if (xs.size() == 3 && perm == Shape{0, 2, 1}) {
    batch = xs[0], rows = xs[1], cols = xs[2];
  } else if (xs.size() == 4 && perm == Shape{0, 2, 3, 1}) {
    batch = xs[0], rows = xs[1], cols = xs[2] * xs[3];
  } else if (xs.size() == 4 && perm == Shape{0, 3, 1, 2}) {
    batch = xs[0], rows = xs[1] * xs[2], cols = xs[3];
  } else if (xs.size() == 4 && perm == Shape{0, 1, 3, 2}) {
    batch = xs[0] * xs[1], rows = xs[2], cols = xs[3];
  }
  if (ops.empty() && a == 0 && xs.size() == 4 && perm == Shape{0, 2, 3, 1})
    input_nhwc_id = y;
  if (batch) {
    add("transpose", [=] {
      check(transpose2d(t[a], t[y], batch, rows, cols, stream), "transpose");
    });
    return;
  }
  if (xs.size() > 6 || perm.size() != xs.size())
    throw std::runtime_error("unsupported transpose rank");
  Gather g;
  g.rank = static_cast<int>(xs.size());
  std::vector<long long> strides(xs.size());
  long long s = 1;
  for (int j = g.rank - 1; j >= 0; --j) {
    strides[j] = s;
    s *= xs[j];
  }
  for (int j = 0; j < g.rank; ++j) {
    g.shape[j] = ys[j];
    g.stride[j] = strides[perm[j]];
  }
  const long long n = count(ys);
  add("gather", [=] { check(gather(t[a], t[y], n, g, stream), "gather"); });
}

void Runtime::slice(int a, int y, Shape xs, Shape ys, Shape starts) {
  reads({a});
  if (xs.size() > 6)
    throw std::runtime_error("unsupported slice rank");
  Gather g;
  g.rank = static_cast<int>(xs.size());
  long long s = 1;
  for (int j = g.rank - 1; j >= 0; --j) {
    g.shape[j] = ys[j];
    g.stride[j] = s;
    g.offset += starts[j] * s;
    s *= xs[j];
  }
  const long long n = count(ys);
  add("slice", [=] { check(gather(t[a], t[y], n, g, stream), "slice"); });
}

void Runtime::concat(int a, int b, int y, int rows, int na, int nb) {
  reads({a, b});
  add("concat", [=] {
    check(concat_rows(t[a], t[b], t[y], rows, na, nb, stream), "concat");
  });
}

void Runtime::pad(int a, int y, Shape xs, Shape ys, int ph, int pw) {
  reads({a});
  add("pad", [=] {
    check(pad_nchw(t[a], t[y], xs[0] * xs[1], xs[2], xs[3], ys[2], ys[3], ph,
                   pw, stream),
          "pad");
  });
}

void Runtime::pad_nhwc(int a, int y, Shape xs, Shape ys, int ph, int pw) {
  reads({a});
  add("pad_nhwc", [=] {
    check(::pb2::pad_nhwc(t[a], t[y], xs[0], xs[1], xs[2], xs[3], ys[2], ys[3],
                          ph, pw, stream),
          "pad_nhwc");
  });
}

void Runtime::pool(int a, int y, Shape xs, Shape ys, Shape k, Shape s, Shape p,
                   bool maximum) {
  reads({a});
  add("pool", [=] {
    check(pool_nchw(t[a], t[y], xs[0] * xs[1], xs[2], xs[3], ys[2], ys[3],
                    k[0], k[1], s[0], s[1], p[0], p[1], maximum, stream),
          "pool");
  });
}

void Runtime::pool_nhwc(int a, int y, Shape xs, Shape ys, Shape k, Shape s,
                        Shape p, bool maximum) {
  reads({a});
  add("pool_nhwc", [=] {
    check(::pb2::pool_nhwc(t[a], t[y], xs[0], xs[1], xs[2], xs[3], ys[2],
                           ys[3], k[0], k[1], s[0], s[1], p[0], p[1], maximum,
                           stream),
          "pool_nhwc");
  });
}

void Runtime::mean(int a, int y, int rows, int cols) {
  reads({a});
  add("mean", [=] {
    check(mean_rows(t[a], t[y], rows, cols, stream), "mean");
  });
}

void Runtime::mean_nhwc(int a, int y, int batch, int channels, int spatial) {
  reads({a});
  add("mean_nhwc", [=] {
    check(::pb2::mean_nhwc(t[a], t[y], batch, channels, spatial, stream),
          "mean_nhwc");
  });
}

void Runtime::resize_nearest(int a, int y, Shape xs, Shape ys, float sh,
                             float sw) {
  reads({a});
  add("resize_nearest", [=] {
    check(resize_nearest_nchw(t[a], t[y], xs[0] * xs[1], xs[2], xs[3], ys[2],
                              ys[3], sh, sw, stream),
          "resize_nearest");
  });
}

void Runtime::resize_nearest_nhwc(int a, int y, Shape xs, Shape ys, float sh,
                                  float sw) {
  reads({a});
  add("resize_nearest_nhwc", [=] {
    check(::pb2::resize_nearest_nhwc(t[a], nullptr, t[y], xs[0], xs[1], xs[2],
                                     xs[3], ys[2], ys[3], sh, sw, stream),
          "resize_nearest_nhwc");
  });
}

void Runtime::upsample_concat_nhwc(std::vector<int> srcs, int y, std::vector<Shape> xs,
                                   Shape ys) {
  if (srcs.empty() || srcs.size() != xs.size() || static_cast<int>(srcs.size()) > pb2::kUpcatMax ||
      ys.size() != 4)
    throw std::runtime_error("upsample_concat_nhwc: 1.." + std::to_string(pb2::kUpcatMax) +
                             " sources with one shape each");
  int ctot = 0;
  for (size_t k = 0; k < srcs.size(); ++k) {
    const Shape &x = xs[k];
    if (x.size() != 4 || x[0] != ys[0] || x[1] % 8 || x[2] <= 0 || x[3] <= 0)
      throw std::runtime_error("upsample_concat_nhwc: source " + std::to_string(k) + " shape " +
                               shape_str(x));
    ctot += x[1];
  }
  if (ctot != ys[1])
    throw std::runtime_error("upsample_concat_nhwc: channels do not add up to " + shape_str(ys));
  for (int id : srcs)
    reads({id});
  add("upsample_concat_nhwc", [=] {
    pb2::UpcatArgs a{};
    a.n = static_cast<int>(srcs.size());
    for (int k = 0; k < a.n; ++k) {
      a.src[k] = t[srcs[k]];
      a.C[k] = xs[k][1];
      a.H[k] = xs[k][2];
      a.W[k] = xs[k][3];
      a.sh[k] = static_cast<float>(ys[2]) / xs[k][2];
      a.sw[k] = static_cast<float>(ys[3]) / xs[k][3];
    }
    check(pb2::upsample_concat_nhwc(a, t[y], ys[0], ys[2], ys[3], stream), "upsample_concat_nhwc");
  });
}

void Runtime::resize_nearest_add_nhwc(int a, int addend, int y, Shape xs,
                                      Shape ys, float sh, float sw) {
  reads({a, addend});
  auto plain = [=] {
    check(::pb2::resize_nearest_nhwc(t[a], t[addend], t[y], xs[0], xs[1],
                                     xs[2], xs[3], ys[2], ys[3], sh, sw,
                                     stream),
          "resize_add_nhwc");
  };
  const PendingGemm m = last_gemm_;
  const int B = xs[0], C = xs[1], H = xs[2], W = xs[3];
  if (m.op >= 0 && m.op == static_cast<int>(ops.size()) - 1 && addend == m.yi && a != m.yi && a != m.ai &&
      sh == 2.f && sw == 2.f && ys[0] == B && ys[1] == C && ys[2] == 2 * H && ys[3] == 2 * W &&
      m.co == C && static_cast<long long>(m.rows) == 4LL * B * H * W && C % 8 == 0 &&
      disjoint(t[m.ai], static_cast<size_t>(m.rows) * m.ci, t[y], static_cast<size_t>(m.rows) * m.co) &&
      disjoint(t[a], static_cast<size_t>(B) * H * W * C, t[y], static_cast<size_t>(m.rows) * m.co)) {
    // FPN step folded into the lateral 1x1 conv that produced the addend:
    // its epilogue adds the nearest-upsampled coarser map and writes y (the
    // same fp16 rounding points: round(lateral) + up(a), rounded).
    reads({a});
    fused_.push_back({m.op, m.yi, ops[m.op], plain, "gemm_epilogue", "resize_add_nhwc"});
    ops[m.op] = [=] {
      GemmEpilogue e;
      e.bias = m.bi >= 0 ? t[m.bi] : nullptr;
      e.residual = t[a];
      e.ldr = C;
      e.res_up = 1;
      e.res_h = H;
      e.res_w = W;
      e.out = t[y];
      e.ldo = m.co;
      e.act = m.act;
      check(tc_gemm(t[m.ai], m.rows, m.ci, m.ci, t[m.wi], m.co, m.ci, e, stream), "tc_gemm");
    };
    op_names.resize(ops.size());
    op_names[m.op] = "gemm_resize_add";
    add_fused_placeholder();
    return;
  }
  add("resize_add_nhwc", plain);
}

void Runtime::attention(int qkv, int y, int lines, int seq, int heads,
                        int head_dim, float scale) {
  reads({qkv});
  add("attention", [=] {
    check(::pb2::attention(t[qkv], t[y], lines, seq, heads, head_dim, scale,
                           stream),
          "attention");
  });
}

void Runtime::run() {
  if (!prepared) {
    for (auto &p : prepare)
      p();
    prepared = true;
  }
  for (size_t i = static_cast<size_t>(first_op); i < ops.size(); ++i)
    ops[i]();
  CU(cudaGetLastError());
}
