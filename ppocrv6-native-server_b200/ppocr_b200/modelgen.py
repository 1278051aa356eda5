"""Synthetic PP-OCR graphs written as `model.inc` + `weights.f32`.

The real PP-OCRv6 ONNX graphs are not available offline, so the benchmark
architectures (arch specs in models/*.json) are emitted directly in the
format tools/compiled_models/export.py writes (export.py:1032-1154):

* `model.inc` defines INPUT_ELEMENTS, OUTPUT_ELEMENTS, OUTPUT_ID,
  MODEL_INPUT_SHAPE, MODEL_OUTPUT_RANK, MODEL_OUTPUT_SHAPE, ARENA_ELEMENTS,
  WEIGHT_ELEMENTS and `template<class ModelRuntime> void build_model(r)`,
  which sets the tensor table `r.t[i]` (weights or arena offsets) and then
  calls the operator API in graph order;
* `weights.f32` is raw little-endian FP32, each tensor padded to a 64-element
  boundary (export.py:1094-1101);
* tensor 0 is the NCHW model input; the first op moves it to channels-last,
  as export.py's channels_last pass does (export.py:577-591);
* convolution filters are stored OHWI (export.py:593-600), depthwise
  [C][KH][KW], linear weights [out][in], BatchNorm is folded into the
  preceding convolution (scale into the filter, shift into the bias).

The emitted op calls use the fused forms the exporter produces for these
patterns (conv/dw + bias + activation, gemm_epilogue for 1x1 and linear
layers with bias, activation and residual), plus the B200 `attention()`
extension for the SVTR mixing block.

Exporter-vocabulary graphs (`Builder(xv=True)`, shapes named `*_xv`) use only
what export.py emits and the reference's Runtime serves, so the same
`model.inc` compiles against both runtimes:
* dense convolutions without bias, followed by the bias add and activation
  as a generated `fused_pointwise_N` kernel (export.py:714-815) -- the
  reference serves those convs with cuDNN, which takes no epilogue;
* depthwise convs of the reference's native shapes and 1x1 convs fuse bias
  and ReLU only (export.py:817-938: codes 0/1); hardswish, sigmoid and swish
  stay in generated kernels (HardSigmoid + Mul, Sigmoid + Mul);
* linear layers as `matmul` on a [in][out] weight plus a generated bias
  (+ residual, + activation) kernel; the attention as reshape/transpose/
  slice, scale `binary_fast`, `matmul` (q.k^T), `softmax`, `matmul` (P.v)
  and a transpose back;
* FPN steps as `resize_nearest_nhwc` + `binary_fast` add and the tail as
  resizes plus a chain of `concat`; transposed convs without bias.
The weights are the same seeded draws in the same order (linear weights
stored transposed), so an `_xv` graph computes the same function as its
fused twin.
"""

from __future__ import annotations

import json
import math
import os
import re
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

ACT = {"none": 0, "relu": 1, "gelu": 2, "hardswish": 3, "sigmoid": 4, "swish": 5, "hardsigmoid": 6}


def vec(v) -> str:
    return "{" + ",".join(str(int(x)) for x in v) + "}"


def flit(value: float) -> str:
    """C++ float literal, formatted like export.py's literal() helper."""
    text = format(float(value), ".9g")
    if "." not in text and "e" not in text:
        text += ".0"
    return text + "f"


@dataclass
class Tensor:
    name: str
    shape: tuple
    const: np.ndarray | None = None
    alias_of: int | None = None  # views share storage with another tensor


@dataclass
class Graph:
    """Tensor table + op list in the export.py model.inc convention."""

    input_shape: tuple
    tensors: list = field(default_factory=list)
    ops: list = field(default_factory=list)  # (inputs, output, code)
    layers: list = field(default_factory=list)  # oracle description
    kernels: list = field(default_factory=list)  # generated __global__ kernels

    def __post_init__(self):
        self.add_tensor("x", self.input_shape)

    def add_tensor(self, name, shape, const=None, alias_of=None) -> int:
        self.tensors.append(Tensor(name, tuple(int(s) for s in shape), const, alias_of))
        return len(self.tensors) - 1

    def const(self, name, value: np.ndarray) -> int:
        return self.add_tensor(name, value.shape, const=np.asarray(value, dtype=np.float32))

    def act(self, name, shape) -> int:
        return self.add_tensor(name, shape)

    def view(self, src: int, name: str, shape) -> int:
        root = src
        while self.tensors[root].alias_of is not None:
            root = self.tensors[root].alias_of
        assert math.prod(shape) == math.prod(self.tensors[src].shape)
        return self.add_tensor(name, shape, alias_of=root)

    def op(self, inputs, output, code, layer=None):
        self.ops.append((list(inputs), output, code))
        if layer is not None:
            self.layers.append(layer)

    # ------------------------------------------------------------- writing
    def _storage(self, i):
        while self.tensors[i].alias_of is not None:
            i = self.tensors[i].alias_of
        return i

    def plan_arena(self, output_id):
        """Best-fit reuse in op order; an op's output never aliases its inputs.

        Mirrors the liveness rule of export.py:1034-1077: the model input and
        output stay live for the whole run.
        """
        n_ops = len(self.ops)
        last = {0: n_ops, self._storage(output_id): n_ops}
        for j, (ins, out, _) in enumerate(self.ops):
            for i in ins:
                s = self._storage(i)
                if self.tensors[s].const is None:
                    last[s] = max(last.get(s, j), j)
            s = self._storage(out)
            last.setdefault(s, j)
        active, free, offsets, high = {}, [], {}, 0

        def size_of(i):
            return (math.prod(self.tensors[i].shape) + 127) // 128 * 128

        def alloc(i, step):
            nonlocal high
            for old, (off, sz) in list(active.items()):
                if last.get(old, -1) < step:
                    free.append((sz, off))
                    del active[old]
            size = size_of(i)
            choices = sorted((sz, off, k) for k, (sz, off) in enumerate(free) if sz >= size)
            if choices:
                sz, off, k = choices[0]
                free.pop(k)
                if sz > size:
                    free.append((sz - size, off + size))
            else:
                off = high
                high += size
            offsets[i] = off
            active[i] = (off, size)

        alloc(0, -1)
        for step, (_, out, _) in enumerate(self.ops):
            s = self._storage(out)
            if s not in offsets:
                alloc(s, step)
        return offsets, high

    def write(self, directory: Path, output_id: int, weights_path: Path | None = None,
              detector: bool = False) -> dict:
        directory.mkdir(parents=True, exist_ok=True)
        offsets, arena = self.plan_arena(output_id)
        out_shape = self.tensors[output_id].shape
        lines = [
            "// Generated by ppocr_b200.modelgen in the export.py model.inc format.",
            *self.kernels,
            f"constexpr size_t INPUT_ELEMENTS = {math.prod(self.input_shape)};",
            f"constexpr size_t OUTPUT_ELEMENTS = {math.prod(out_shape)};",
            f"constexpr int OUTPUT_ID = {output_id};",
            f"constexpr int MODEL_INPUT_SHAPE[4] = {vec(self.input_shape)};",
            f"constexpr int MODEL_OUTPUT_RANK = {len(out_shape)};",
            f"constexpr int MODEL_OUTPUT_SHAPE[4] = {vec(list(out_shape) + [1] * (4 - len(out_shape)))};",
            f"constexpr size_t ARENA_ELEMENTS = {arena};",
            "template<class ModelRuntime> void build_model(ModelRuntime& r) {",
            f"r.t.resize({len(self.tensors)});",
        ]
        offset = 0
        consts = []
        for i, t in enumerate(self.tensors):
            if t.const is not None:
                pad = (-offset) % 64
                offset += pad
                consts.append((pad, t.const))
                lines.append(f"r.t[{i}] = r.weights + {offset};")
                offset += t.const.size
            else:
                # Tensors no op produces (a truncated graph) get offset 0.
                lines.append(f"r.t[{i}] = r.arena + {offsets.get(self._storage(i), 0)};")
        for _, _, code in self.ops:
            # build_model is a template: member templates need `template`.
            lines.append(re.sub(r"r\.(\w+)<", r"r.template \1<", code))
        lines.append("}")
        lines.append(f"constexpr size_t WEIGHT_ELEMENTS = {offset};")
        (directory / "model.inc").write_text("\n".join(lines) + "\n")
        if detector:
            (directory / "DETECTOR").write_text("1\n")
        if weights_path is not None:
            write_weights(weights_path, consts)
        meta = {
            "input_shape": list(self.input_shape),
            "output_shape": list(out_shape),
            "output_id": output_id,
            "arena_elements": arena,
            "weight_elements": offset,
            "operations": len(self.ops),
        }
        return meta

    def weight_consts(self):
        offset = 0
        consts = []
        for t in self.tensors:
            if t.const is not None:
                pad = (-offset) % 64
                offset += pad
                consts.append((pad, t.const))
                offset += t.const.size
        return consts, offset


def write_weights(path: Path, consts) -> None:
    """Writes atomically: several processes (one per GPU) may generate the
    same deterministic file at once; each renames its own temporary."""
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(f".tmp{os.getpid()}")
    with tmp.open("wb") as f:
        for pad, v in consts:
            if pad:
                f.write(bytes(pad * 4))
            f.write(np.ascontiguousarray(v, dtype="<f4").tobytes())
    tmp.replace(path)


# ------------------------------------------------------------------ builders
class Init:
    """Seeded weight initialisation (numpy PCG64)."""

    def __init__(self, seed: int):
        self.rng = np.random.default_rng(seed)

    def he(self, shape, fan_in):
        return (self.rng.standard_normal(shape) * math.sqrt(2.0 / fan_in)).astype(np.float32)

    def xavier(self, shape, fan_in, fan_out):
        a = math.sqrt(6.0 / (fan_in + fan_out))
        return self.rng.uniform(-a, a, shape).astype(np.float32)

    def normal(self, shape, mean, std):
        return (mean + std * self.rng.standard_normal(shape)).astype(np.float32)


# Depthwise shapes the reference serves with its own kernels (and so with a
# fused bias + activation): runtime.cuh:668-765, export.py:855-866.
def _native_dw(kh, kw, stride) -> bool:
    stride = list(stride)
    return ((kh, kw) == (3, 3) and stride in ([1, 1], [2, 1], [2, 2])) or \
        ((kh, kw) == (9, 9) and stride == [1, 1]) or ((kh, kw) == (1, 7) and stride == [1, 1])


# Activations the exporter fuses into gemm_epilogue / a depthwise conv
# (export.py:878-909 codes 0 bias, 1 ReLU; GELU is not used here).
_FUSABLE = ("none", "relu")


class Builder:
    """Emits layers into a Graph and records an oracle layer description.

    With xv=True the graph is written in the exporter's own vocabulary
    (module docstring); no oracle layer description is recorded then."""

    def __init__(self, g: Graph, init: Init, xv: bool = False):
        self.g = g
        self.init = init
        self.n = 0
        self.xv = xv

    def _name(self, kind):
        self.n += 1
        return f"{kind}_{self.n}"

    def _layer(self, layer):
        return None if self.xv else layer

    # ------------------------------------------------- exporter vocabulary
    @staticmethod
    def _index(src_shape, dst_shape) -> str:
        """flat_index<D,M> of a contiguous broadcast (export.py
        flat_broadcast): same size, a per-channel vector over channels-last
        data, or a scalar."""
        n, m = math.prod(dst_shape), math.prod(src_shape)
        if m == n:
            return "flat_index<1,0>(i)"
        if m == 1:
            return "flat_index<1,1>(i)"
        assert m == dst_shape[-1], (src_shape, dst_shape)
        return f"flat_index<1,{m}>(i)"

    def ew(self, name, out_shape, inputs, body, op_layer=None) -> int:
        """A generated elementwise kernel in the exporter's fused_pointwise
        form: `body` lists expressions over a0..ak (the inputs, loaded as
        float) and v0..v(j-1) (earlier values); the last value is stored."""
        g = self.g
        y = g.act(name, out_shape)
        n = math.prod(out_shape)
        k = len(g.kernels)
        params = ",".join([f"const Scalar* p{j}" for j in range(len(inputs))] + ["Scalar* y"])
        loads = {f"a{j}": f"float(p{j}[{self._index(g.tensors[t].shape, out_shape)}])"
                 for j, t in enumerate(inputs)}
        text = []
        for j, expr in enumerate(body):
            for key, val in loads.items():
                expr = re.sub(rf"\b{key}\b", val, expr)
            text.append(f"  float v{j} = {expr};")
        g.kernels.append(
            f"__global__ void fused_pointwise_{k}({params}) {{\n"
            f"  int i=blockIdx.x*blockDim.x+threadIdx.x;if(i>={n})return;\n"
            + "\n".join(text) + f"\n  y[i]=v{len(body) - 1};\n}}")
        args = ",".join(f"r.t[{t}]" for t in list(inputs) + [y])
        g.op(list(inputs), y,
             f"r.ops.emplace_back([&r]{{fused_pointwise_{k}<<<{(n + 255) // 256},256,0,r.stream>>>({args});}});",
             op_layer)
        return y

    def bias_act_xv(self, x, bias, act, residual=-1, name=None):
        """The exporter's lowering of `+ bias [+ residual] [activation]`:
        one binary_fast when the bias add stands alone, otherwise one
        generated kernel (values stay fp32 inside it)."""
        g = self.g
        shape = g.tensors[x].shape
        name = name or self._name("bias")
        n = math.prod(shape)
        if residual < 0 and act == "none":
            y = g.act(name, shape)
            g.op([x, bias], y, f"r.binary_fast<0,1,0,1,{shape[-1]}>({x},{bias},{y},{n});")
            return y
        ins = [x, bias] + ([residual] if residual >= 0 else [])
        body = ["(a0 + a1)"]
        if residual >= 0:
            body.append("(v0 + a2)")
        v = f"v{len(body) - 1}"
        if act == "relu":
            body.append(f"fmaxf({v},0.f)")
        elif act == "sigmoid":
            body.append(f"(1.f/(1.f+expf(-({v}))))")
        elif act == "hardswish":
            body.append(f"fminf(1.f,fmaxf(0.f,({flit(np.float32(1.0 / 6.0))})*({v})+(0.5f)))")
            body.append(f"({v} * v{len(body) - 1})")
        elif act == "swish":
            body.append(f"(1.f/(1.f+expf(-({v}))))")
            body.append(f"({v} * v{len(body) - 1})")
        else:
            assert act == "none", act
        return self.ew(name, shape, ins, body)

    def to_nhwc(self, x):
        b, c, h, w = self.g.tensors[x].shape
        y = self.g.act("x_nhwc", (b, h, w, c))
        self.g.op([x], y, f"r.transpose({x},{y},{vec((b, c, h, w))},{vec((b, h, w, c))},{{0,2,3,1}});",
                  self._layer({"op": "to_nhwc", "in": x, "out": y}))
        return y

    def conv_bn_act(self, x, co, k, stride=(1, 1), act="relu", depthwise=False):
        """Conv (+ folded BN) + activation on an NHWC tensor (logical NCHW args)."""
        b, h, w, c = self.g.tensors[x].shape
        kh, kw = (k, k) if isinstance(k, int) else k
        ph, pw = kh // 2, kw // 2
        oh = (h + 2 * ph - kh) // stride[0] + 1
        ow = (w + 2 * pw - kw) // stride[1] + 1
        name = self._name("dw" if depthwise else "conv")
        if depthwise:
            assert co == c
            wshape = (c, 1, kh, kw)
            wt = self.init.he((c, kh, kw), kh * kw)
            groups = c
        else:
            wshape = (co, c, kh, kw)
            wt = self.init.he((co, kh, kw, c), kh * kw * c)
            groups = 1
        scale = self.init.normal((co,), 1.0, 0.1)
        shift = self.init.normal((co,), 0.0, 0.1)
        wt = wt * scale.reshape((co,) + (1,) * (wt.ndim - 1))
        wi = self.g.const(name + "_w", wt)
        bi = self.g.const(name + "_b", shift)
        args = (f"{vec((b, c, h, w))},{vec(wshape)},{vec((b, co, oh, ow))},{vec((ph, pw))},{vec(stride)},"
                f"{{1,1}},{groups},true,true")
        if self.xv and not (depthwise and _native_dw(kh, kw, stride) and act in _FUSABLE):
            # cuDNN in the reference: no epilogue; bias + activation follow.
            yc = self.g.act(name + "_before_bias", (b, oh, ow, co))
            self.g.op([x, wi], yc, f"r.conv({x},{wi},{yc},{args});")
            return self.bias_act_xv(yc, bi, act, name=name)
        y = self.g.act(name, (b, oh, ow, co))
        self.g.op([x, wi, bi], y, f"r.conv({x},{wi},{y},{args},{bi},{ACT[act]});",
                  self._layer({"op": "conv", "in": x, "w": wi, "b": bi, "out": y, "stride": list(stride),
                               "pad": [ph, pw], "groups": groups, "act": ACT[act]}))
        return y

    def pointwise(self, x, co, act="relu"):
        """1x1 conv + folded BN + activation as the exporter's gemm_epilogue."""
        b, h, w, c = self.g.tensors[x].shape
        name = self._name("pw")
        wt = self.init.he((co, c), c)
        scale = self.init.normal((co,), 1.0, 0.1)
        shift = self.init.normal((co,), 0.0, 0.1)
        wi = self.g.const(name + "_w", wt * scale[:, None])
        bi = self.g.const(name + "_b", shift)
        rows = b * h * w
        if self.xv and act not in _FUSABLE:
            # A 1x1 conv whose epilogue the exporter cannot fuse
            # (cublasGemmEx in the reference), then a generated kernel.
            yc = self.g.act(name + "_before_bias", (b, h, w, co))
            self.g.op([x, wi], yc, f"r.conv({x},{wi},{yc},{vec((b, c, h, w))},{vec((co, c, 1, 1))},"
                                   f"{vec((b, co, h, w))},{{0,0}},{{1,1}},{{1,1}},1,true,true);")
            return self.bias_act_xv(yc, bi, act, name=name)
        y = self.g.act(name, (b, h, w, co))
        self.g.op([x, wi, bi], y, f"r.gemm_epilogue({x},{wi},{bi},-1,{y},{rows},{c},{co},{ACT[act]});",
                  self._layer({"op": "gemm", "in": x, "w": wi, "b": bi, "res": -1, "out": y, "act": ACT[act]}))
        return y

    def linear(self, x, co, act="none", residual=-1, bias_std=0.01):
        shape = self.g.tensors[x].shape
        c = shape[-1]
        rows = math.prod(shape[:-1])
        name = self._name("linear")
        wt = self.init.xavier((co, c), c, co)
        if self.xv:
            # ONNX MatMul right-hand side [in][out] -> Runtime::matmul, then
            # the bias (+ residual, + activation) as a generated kernel.
            wi = self.g.const(name + "_w", np.ascontiguousarray(wt.T))
            bi = self.g.const(name + "_b", self.init.normal((co,), 0.0, bias_std))
            ym = self.g.act(name + "_matmul", shape[:-1] + (co,))
            self.g.op([x, wi], ym, f"r.matmul({x},{wi},{ym},1,{rows},{co},{c});")
            return self.bias_act_xv(ym, bi, act, residual, name=name)
        wi = self.g.const(name + "_w", wt)
        bi = self.g.const(name + "_b", self.init.normal((co,), 0.0, bias_std))
        y = self.g.act(name, shape[:-1] + (co,))
        self.g.op([x, wi, bi] + ([residual] if residual >= 0 else []), y,
                  f"r.gemm_epilogue({x},{wi},{bi},{residual},{y},{rows},{c},{co},{ACT[act]});",
                  self._layer({"op": "gemm", "in": x, "w": wi, "b": bi, "res": residual, "out": y,
                               "act": ACT[act]}))
        return y

    def layernorm(self, x, eps=1e-6):
        shape = self.g.tensors[x].shape
        c = shape[-1]
        rows = math.prod(shape[:-1])
        name = self._name("ln")
        si = self.g.const(name + "_scale", self.init.normal((c,), 1.0, 0.05))
        bi = self.g.const(name + "_bias", self.init.normal((c,), 0.0, 0.05))
        y = self.g.act(name, shape)
        self.g.op([x, si, bi], y, f"r.layernorm({x},{si},{bi},{y},{rows},{c},{flit(eps)});",
                  self._layer({"op": "layernorm", "in": x, "scale": si, "bias": bi, "out": y, "eps": eps}))
        return y

    def attention(self, qkv, heads, head_dim):
        lines, seq, width = self.g.tensors[qkv].shape
        assert width == 3 * heads * head_dim
        scale = head_dim ** -0.5
        if self.xv:
            return self._attention_xv(qkv, heads, head_dim, scale)
        y = self.g.act(self._name("attn"), (lines, seq, heads * head_dim))
        self.g.op([qkv], y, f"r.attention({qkv},{y},{lines},{seq},{heads},{head_dim},{flit(scale)});",
                  {"op": "attention", "in": qkv, "out": y, "heads": heads, "dh": head_dim,
                   "scale": float(np.float32(scale))})
        return y

    def _attention_xv(self, qkv, heads, dh, scale):
        """SVTR attention as the exporter lowers the ONNX graph: reshape
        [L,T,3,h,dh] -> transpose (2,0,3,1,4) -> slices q/k/v -> q*scale ->
        matmul(q, k^T) -> softmax -> matmul(P, v) -> transpose (0,2,1,3)."""
        g = self.g
        L, T, _ = g.tensors[qkv].shape
        name = self._name("attn")
        v5 = g.view(qkv, name + "_qkv5", (L, T, 3, heads, dh))
        tr = g.act(name + "_perm", (3, L, heads, T, dh))
        g.op([v5], tr, f"r.transpose({v5},{tr},{vec((L, T, 3, heads, dh))},{vec((3, L, heads, T, dh))},"
                       f"{{2,0,3,1,4}});")
        parts = []
        for j, part in enumerate("qkv"):
            sl = g.act(f"{name}_{part}", (1, L, heads, T, dh))
            g.op([tr], sl, f"r.slice({tr},{sl},{vec((3, L, heads, T, dh))},{vec((1, L, heads, T, dh))},"
                           f"{vec((j, 0, 0, 0, 0))});")
            parts.append(g.view(sl, f"{name}_{part}4", (L, heads, T, dh)))
        q, k, v = parts
        sc = g.const(name + "_scale", np.array([scale], np.float32))
        qs = g.act(name + "_qs", (L, heads, T, dh))
        n = L * heads * T * dh
        g.op([q, sc], qs, f"r.binary_fast<2,1,0,1,1>({q},{sc},{qs},{n});")
        kt = g.act(name + "_kt", (L, heads, dh, T))
        g.op([k], kt, f"r.transpose({k},{kt},{vec((L, heads, T, dh))},{vec((L, heads, dh, T))},{{0,1,3,2}});")
        s_ = g.act(name + "_scores", (L, heads, T, T))
        g.op([qs, kt], s_, f"r.matmul({qs},{kt},{s_},{L * heads},{T},{T},{dh});")
        pr = g.act(name + "_probs", (L, heads, T, T))
        g.op([s_], pr, f"r.softmax({s_},{pr},{L * heads * T},{T});")
        o = g.act(name + "_o", (L, heads, T, dh))
        g.op([pr, v], o, f"r.matmul({pr},{v},{o},{L * heads},{T},{dh},{T});")
        ot = g.act(name + "_ot", (L, T, heads, dh))
        g.op([o], ot, f"r.transpose({o},{ot},{vec((L, heads, T, dh))},{vec((L, T, heads, dh))},{{0,2,1,3}});")
        return g.view(ot, name, (L, T, heads * dh))

    def avgpool(self, x, k, s):
        b, h, w, c = self.g.tensors[x].shape
        oh, ow = (h - k[0]) // s[0] + 1, (w - k[1]) // s[1] + 1
        y = self.g.act(self._name("pool"), (b, oh, ow, c))
        self.g.op([x], y, f"r.pool_nhwc({x},{y},{vec((b, c, h, w))},{vec((b, c, oh, ow))},"
                          f"{vec(k)},{vec(s)},{{0,0}},false);",
                  self._layer({"op": "avgpool", "in": x, "out": y, "k": list(k), "s": list(s)}))
        return y


def svtr_block(bd: Builder, x, heads, head_dim, mlp_ratio=2):
    dim = bd.g.tensors[x].shape[-1]
    h = bd.layernorm(x)
    qkv = bd.linear(h, 3 * dim)
    att = bd.attention(qkv, heads, head_dim)
    x = bd.linear(att, dim, residual=x)
    h = bd.layernorm(x)
    f = bd.linear(h, dim * mlp_ratio, act="swish")
    return bd.linear(f, dim, residual=x)


def build_recognizer(spec: dict, batch: int, seed: int, xv: bool = False):
    """HGNet-style backbone + SVTR neck; output hidden [B, T, dim]."""
    height, width = spec["height"], spec["width"]
    g = Graph((batch, 3, height, width))
    bd = Builder(g, Init(seed), xv)
    x = bd.to_nhwc(0)
    stem = spec["stem"]
    x = bd.conv_bn_act(x, stem[0], 3, stride=(2, 2))
    for co in stem[1:]:
        x = bd.conv_bn_act(x, co, 3)
    for st in spec["stages"]:
        c = g.tensors[x].shape[-1]
        x = bd.conv_bn_act(x, c, 3, stride=tuple(st["stride"]), depthwise=True)
        x = bd.conv_bn_act(x, st["out"], 3)
        x = bd.pointwise(x, st["out"])
    x = bd.avgpool(x, tuple(spec["pool"]), tuple(spec["pool"]))
    b, h, w, c = g.tensors[x].shape
    assert h == 1
    seq = g.view(x, "sequence", (b, w, c))
    neck = spec["neck"]
    x = bd.linear(seq, neck["dim"])
    for _ in range(neck["blocks"]):
        x = svtr_block(bd, x, neck["heads"], neck["dim"] // neck["heads"], neck.get("mlp_ratio", 2))
    return g, x


def build_block(spec: dict, batch: int, seed: int, xv: bool = False):
    """Depthwise-separable NHWC block: dw KxK (+BN, act) -> 1x1 (+BN, act)."""
    g = Graph((batch, spec["channels"], spec["height"], spec["width"]))
    bd = Builder(g, Init(seed), xv)
    x = bd.to_nhwc(0)
    c = spec["channels"]
    x = bd.conv_bn_act(x, c, spec["kernel"], act=spec["act"], depthwise=True)
    x = bd.pointwise(x, spec["out"], act=spec["act"])
    return g, x


def build_neck(spec: dict, batch: int, seed: int, xv: bool = False):
    """SVTR neck alone on [B, seq, dim] FP16 tokens (input viewed as
    [B, 1, seq, dim], where NCHW and NHWC coincide)."""
    seq, dim = spec["seq"], spec["dim"]
    g = Graph((batch, 1, seq, dim))
    bd = Builder(g, Init(seed), xv)
    x = g.view(0, "tokens", (batch, seq, dim))
    for _ in range(spec["blocks"]):
        x = svtr_block(bd, x, spec["heads"], dim // spec["heads"], spec.get("mlp_ratio", 2))
    return g, x


def _move_op_before(g: Graph, src_out: int, dst_out: int) -> None:
    """Moves the op writing src_out (and its layer record) to just before the
    op writing dst_out; ops and layers are aligned one to one here."""
    assert len(g.ops) == len(g.layers)
    i = next(k for k, op in enumerate(g.ops) if op[1] == src_out)
    op, layer = g.ops.pop(i), g.layers.pop(i)
    j = next(k for k, o in enumerate(g.ops) if o[1] == dst_out)
    g.ops.insert(j, op)
    g.layers.insert(j, layer)


def build_detector(spec: dict, batch: int, size: int, seed: int, fused_fpn_tail: bool = True,
                   xv: bool = False):
    """Backbone at strides 2..32 + FPN(256) + DB head -> sigmoid map [B,1,S,S]."""
    g = Graph((batch, 3, size, size))
    bd = Builder(g, Init(seed), xv)
    fused_fpn_tail = fused_fpn_tail and not xv
    x = bd.to_nhwc(0)
    stem = spec["stem"]
    x = bd.conv_bn_act(x, stem[0], 3, stride=(2, 2))
    for co in stem[1:]:
        x = bd.conv_bn_act(x, co, 3)
    feats = []
    for st in spec["stages"]:
        c = g.tensors[x].shape[-1]
        x = bd.conv_bn_act(x, c, 3, stride=tuple(st["stride"]), depthwise=True)
        x = bd.conv_bn_act(x, st["out"], 3)
        x = bd.pointwise(x, st["out"])
        feats.append(x)
    fpn = spec["fpn"]
    lat = [bd.pointwise(f, fpn, act="none") for f in feats]
    # Top-down nearest-upsample-add.
    td = [None] * len(lat)
    td[-1] = lat[-1]
    for i in range(len(lat) - 2, -1, -1):
        b, h, w, c = g.tensors[lat[i]].shape
        _, hs, ws_, _ = g.tensors[td[i + 1]].shape
        sh, sw = h / hs, w / ws_
        if xv:
            up = g.act(bd._name("fpn_up"), (b, h, w, c))
            g.op([td[i + 1]], up, f"r.resize_nearest_nhwc({td[i + 1]},{up},{vec((b, c, hs, ws_))},"
                                  f"{vec((b, c, h, w))},{flit(sh)},{flit(sw)});")
            y = g.act(bd._name("fpn_add"), (b, h, w, c))
            g.op([up, lat[i]], y, f"r.binary_fast<0,1,0,1,0>({up},{lat[i]},{y},{b * h * w * c});")
            td[i] = y
            continue
        y = g.act(bd._name("fpn_add"), (b, h, w, c))
        g.op([td[i + 1], lat[i]], y,
             f"r.resize_nearest_add_nhwc({td[i + 1]},{lat[i]},{y},{vec((b, c, hs, ws_))},{vec((b, c, h, w))},"
             f"{flit(sh)},{flit(sw)});",
             {"op": "resize_add", "in": td[i + 1], "add": lat[i], "out": y, "scale": [sh, sw]})
        td[i] = y
    if not xv:
        # Each lateral 1x1 conv runs right before the resize-add that reads
        # it (same weights, drawn in level order above), so the Runtime can
        # fold the add into the conv's epilogue (the exporter keeps its own
        # order in the `_xv` twin).
        for i in range(len(lat) - 1):
            _move_op_before(g, lat[i], td[i])
    outs = [bd.conv_bn_act(t, fpn // 4, 3, act="none") for t in td]
    # Upsample each level to the finest and concatenate channels. The
    # exporter writes this as one Resize per level and a chain of Concats;
    # with fused_fpn_tail the graph carries the Runtime extension that does
    # both in one pass (the same values; no intermediate tensors).
    b, h0, w0, c0 = g.tensors[outs[0]].shape
    if fused_fpn_tail:
        shapes = [g.tensors[o].shape for o in outs]
        ctot = sum(sh[-1] for sh in shapes)
        cat = g.act(bd._name("upcat"), (b, h0, w0, ctot))
        srcs = "{" + ",".join(str(o) for o in outs) + "}"
        xs = "{" + ",".join(vec((b, sh[3], sh[1], sh[2])) for sh in shapes) + "}"
        g.op(list(outs), cat, f"r.upsample_concat_nhwc({srcs},{cat},{xs},{vec((b, ctot, h0, w0))});",
             {"op": "upsample_concat", "in": list(outs), "out": cat})
    else:
        ups = [outs[0]]
        for o in outs[1:]:
            _, h, w, c = g.tensors[o].shape
            y = g.act(bd._name("up"), (b, h0, w0, c))
            g.op([o], y, f"r.resize_nearest_nhwc({o},{y},{vec((b, c, h, w))},{vec((b, c, h0, w0))},"
                         f"{flit(h0 / h)},{flit(w0 / w)});",
                 bd._layer({"op": "resize", "in": o, "out": y, "scale": [h0 / h, w0 / w]}))
            ups.append(y)
        cat = ups[0]
        width = c0
        for u in ups[1:]:
            cu = g.tensors[u].shape[-1]
            y = g.act(bd._name("cat"), (b, h0, w0, width + cu))
            g.op([cat, u], y, f"r.concat({cat},{u},{y},{b * h0 * w0},{width},{cu});",
                 bd._layer({"op": "concat", "a": cat, "b": u, "out": y}))
            cat, width = y, width + cu
    head = spec["head"]
    x = bd.conv_bn_act(cat, head, 3)
    for i, (co, act) in enumerate([(head, "relu"), (1, "sigmoid")]):
        b, h, w, c = g.tensors[x].shape
        name = bd._name("deconv")
        wt = bd.init.he((c, 2, 2, co), c * 4)
        if act == "relu":
            scale = bd.init.normal((co,), 1.0, 0.1)
            wt = wt * scale.reshape(1, 1, 1, co)
            bias = bd.init.normal((co,), 0.0, 0.1)
        else:
            bias = bd.init.normal((co,), 0.0, 0.1)
        wi = g.const(name + "_w", wt)
        bi = g.const(name + "_b", bias)
        if xv:
            # cuDNN backward-data in the reference: no bias, no activation.
            yd = g.act(name + "_before_bias", (b, 2 * h, 2 * w, co))
            g.op([x, wi], yd, f"r.deconv({x},{wi},{yd},{vec((b, c, h, w))},{vec((c, co, 2, 2))},"
                              f"{vec((b, co, 2 * h, 2 * w))},{{0,0}},{{2,2}},{{1,1}},true);")
            x = bd.bias_act_xv(yd, bi, act, name=name)
            continue
        y = g.act(name, (b, 2 * h, 2 * w, co))
        g.op([x, wi, bi], y,
             f"r.deconv({x},{wi},{y},{vec((b, c, h, w))},{vec((c, co, 2, 2))},{vec((b, co, 2 * h, 2 * w))},"
             f"{{0,0}},{{2,2}},{{1,1}},true,{bi},{ACT[act]});",
             {"op": "deconv", "in": x, "w": wi, "b": bi, "out": y, "act": ACT[act]})
        x = y
    b, h, w, _ = g.tensors[x].shape
    out = g.view(x, "maps", (b, 1, h, w))
    return g, out


def build_fusion_probe(seed: int, split: bool, batch: int = 2, size: int = 16):
    """Test graph for the Runtime's speculative fusions: a depthwise conv +
    pointwise GEMM pair (fused block), a lateral 1x1 GEMM + nearest 2x
    resize-add (upsampled residual in the GEMM epilogue) and the DB head's
    two transposed convs (fused tail), chained. With split=True a later op
    reads each pair's intermediate (its output feeds nothing), so every pair
    must split back into its two ops; the chain's output is the same. The
    pairs' inputs are read again at the end in both variants."""
    g = Graph((batch, 3, size, size))
    bd = Builder(g, Init(seed))
    side = Init(seed + 1)  # the split readers' weights: the chain draws the same values either way

    def read_later(t):
        main, bd.init = bd.init, side
        bd.pointwise(t, 64, act="none")
        bd.init = main

    x = bd.to_nhwc(0)
    c1 = bd.conv_bn_act(x, 64, 3)
    # dw 3x3 + pw: the fused depthwise + pointwise block
    d = bd.conv_bn_act(c1, 64, 3, depthwise=True)
    pw = bd.pointwise(d, 64)
    if split:
        read_later(d)
    # lateral 1x1 + resize-add of a coarser map
    coarse = bd.conv_bn_act(pw, 64, 3, stride=(2, 2), depthwise=True)
    lat = bd.pointwise(pw, 64, act="none")
    b, h, w, c = g.tensors[lat].shape
    _, hs, ws_, _ = g.tensors[coarse].shape
    y = g.act(bd._name("fpn_add"), (b, h, w, c))
    g.op([coarse, lat], y,
         f"r.resize_nearest_add_nhwc({coarse},{lat},{y},{vec((b, c, hs, ws_))},{vec((b, c, h, w))},"
         f"{flit(h / hs)},{flit(w / ws_)});",
         {"op": "resize_add", "in": coarse, "add": lat, "out": y, "scale": [h / hs, w / ws_]})
    if split:
        read_later(lat)
    # DB tail: deconv 64 -> 64 (+ReLU) then 64 -> 1 (+sigmoid)
    x = y
    first = None
    for co, act in ((64, "relu"), (1, "sigmoid")):
        b, h, w, c = g.tensors[x].shape
        name = bd._name("deconv")
        wi = g.const(name + "_w", bd.init.he((c, 2, 2, co), c * 4))
        bi = g.const(name + "_b", bd.init.normal((co,), 0.0, 0.1))
        yd = g.act(name, (b, 2 * h, 2 * w, co))
        g.op([x, wi, bi], yd,
             f"r.deconv({x},{wi},{yd},{vec((b, c, h, w))},{vec((c, co, 2, 2))},{vec((b, co, 2 * h, 2 * w))},"
             f"{{0,0}},{{2,2}},{{1,1}},true,{bi},{ACT[act]});",
             {"op": "deconv", "in": x, "w": wi, "b": bi, "out": yd, "act": ACT[act]})
        first = yd if first is None else first
        x = yd
    if split:
        read_later(first)
    # Keep every pair's input alive to the end, so the arena planner cannot
    # hand a pair's output the space of its dying input (the Runtime fuses
    # only when the fused kernel's input and output are disjoint).
    for t in (c1, pw, y):
        read_later(t)
    b, h, w, _ = g.tensors[x].shape
    return g, g.view(x, "maps", (b, 1, h, w))


# Segments of the operator zoo's output, in order: (name, shape).
ZOO_INPUT = (2, 8, 12, 16)


def build_zoo_xv(seed: int):
    """Operator zoo in the exporter's vocabulary: one graph that runs every
    Runtime method the benchmark graphs do not (NCHW pad / pool / nearest
    resize / mean, the six unary modes, general-broadcast binary ops, the
    transpose and concat forms, slices, pad_nhwc, both pool_nhwc fast forms,
    both mean_nhwc forms, batched matmul on constant and computed operands)
    and concatenates every result, flattened, into the output vector.

    Returns (graph, output id, segments) where segments lists each result's
    (name, shape) in output order."""
    B, C, H, W = ZOO_INPUT
    g = Graph(ZOO_INPUT)
    init = Init(seed)
    results = []

    def act(name, shape):
        return g.act(name, shape)

    def op(ins, y, code, name):
        g.op(ins, y, code)
        results.append((name, y))
        return y

    n = B * C * H * W
    x = 0
    # NCHW operators on the staged input (tensor 0 stays NCHW: the first op
    # is not the channels-last transpose).
    p = op([x], act("pad", (B, C, H + 2, W + 2)),
           f"r.pad({x},{{y}},{vec(ZOO_INPUT)},{vec((B, C, H + 2, W + 2))},1,1);", "pad")
    pm = op([p], act("pool_max", (B, C, H, W)),
            f"r.pool({p},{{y}},{vec((B, C, H + 2, W + 2))},{vec((B, C, H, W))},{{3,3}},{{1,1}},{{0,0}},true);",
            "pool_max")
    pa = op([x], act("pool_avg", (B, C, 6, 8)),
            f"r.pool({x},{{y}},{vec(ZOO_INPUT)},{vec((B, C, 6, 8))},{{3,3}},{{2,2}},{{1,1}},false);", "pool_avg")
    op([pa], act("resize", (B, C, H, W)),
       f"r.resize_nearest({pa},{{y}},{vec((B, C, 6, 8))},{vec((B, C, H, W))},2.0f,2.0f);", "resize")
    op([x], act("mean", (B * C,)), f"r.mean({x},{{y}},{B * C},{H * W});", "mean")
    unary = {}
    for mode, (alpha, beta) in enumerate([(0.2, 0.5)] * 6):
        src = unary.get(1, x) if mode == 4 else x  # sqrt of the sigmoid output (positive)
        unary[mode] = op([src], act(f"unary{mode}", ZOO_INPUT),
                         f"r.unary({src},{{y}},{n},{mode},{flit(alpha)},{flit(beta)});", f"unary{mode}")
    chan = g.const("chan", init.normal((1, C, 1, 1), 1.0, 0.3))
    rowc = g.const("rowc", init.normal((B, 1, H, 1), 0.0, 0.5))
    expo = g.const("expo", init.rng.uniform(0.5, 2.0, (1, C, 1, 1)).astype(np.float32))
    for mode in range(4):
        op([x, chan], act(f"binary{mode}", ZOO_INPUT),
           f"r.binary({x},{chan},{{y}},{vec(ZOO_INPUT)},{vec((1, C, 1, 1))},{vec(ZOO_INPUT)},{mode});",
           f"binary{mode}")
    op([unary[1], expo], act("binary4", ZOO_INPUT),
       f"r.binary({unary[1]},{expo},{{y}},{vec(ZOO_INPUT)},{vec((1, C, 1, 1))},{vec(ZOO_INPUT)},4);", "binary4")
    op([x, rowc], act("binary_rows", ZOO_INPUT),
       f"r.binary({x},{rowc},{{y}},{vec(ZOO_INPUT)},{vec((B, 1, H, 1))},{vec(ZOO_INPUT)},2);", "binary_rows")
    op([x], act("transpose_0132", (B, C, W, H)),
       f"r.transpose({x},{{y}},{vec(ZOO_INPUT)},{vec((B, C, W, H))},{{0,1,3,2}});", "transpose_0132")
    op([x], act("slice", (B, 4, 6, 10)),
       f"r.slice({x},{{y}},{vec(ZOO_INPUT)},{vec((B, 4, 6, 10))},{{0,2,3,4}});", "slice")
    # Channels-last operators.
    t = op([x], act("nhwc", (B, H, W, C)),
           f"r.transpose({x},{{y}},{vec(ZOO_INPUT)},{vec((B, H, W, C))},{{0,2,3,1}});", "nhwc")
    op([t], act("pad_nhwc", (B, H + 4, W + 4, C)),
       f"r.pad_nhwc({t},{{y}},{vec(ZOO_INPUT)},{vec((B, C, H + 4, W + 4))},2,2);", "pad_nhwc")
    op([t], act("pool_nhwc_max", (B, H - 1, W - 1, C)),
       f"r.pool_nhwc({t},{{y}},{vec(ZOO_INPUT)},{vec((B, C, H - 1, W - 1))},{{2,2}},{{1,1}},{{0,0}},true);",
       "pool_nhwc_max")
    op([t], act("pool_nhwc_avg", (B, H // 3, W // 2, C)),
       f"r.pool_nhwc({t},{{y}},{vec(ZOO_INPUT)},{vec((B, C, H // 3, W // 2))},{{3,2}},{{3,2}},{{0,0}},false);",
       "pool_nhwc_avg")
    op([t], act("mean_nhwc", (B, C)), f"r.mean_nhwc({t},{{y}},{B},{C},{H * W});", "mean_nhwc")
    big = op([t], act("resize_nhwc", (B, 4 * H, 4 * W, C)),
             f"r.resize_nearest_nhwc({t},{{y}},{vec(ZOO_INPUT)},{vec((B, C, 4 * H, 4 * W))},4.0f,4.0f);",
             "resize_nhwc")
    op([big], act("mean_nhwc_chunked", (B, C)), f"r.mean_nhwc({big},{{y}},{B},{C},{16 * H * W});",
       "mean_nhwc_chunked")
    c16 = op([t, t], act("concat_vec8", (B, H, W, 2 * C)),
             f"r.concat({t},{t},{{y}},{B * H * W},{C},{C});", "concat_vec8")
    op([c16], act("transpose_tiled", (B, 2 * C, H, W)),
       f"r.transpose({c16},{{y}},{vec((B, H, W, 2 * C))},{vec((B, 2 * C, H, W))},{{0,3,1,2}});", "transpose_tiled")
    s3 = op([t], act("slice3", (B, H, W, 3)),
            f"r.slice({t},{{y}},{vec((B, H, W, C))},{vec((B, H, W, 3))},{{0,0,0,0}});", "slice3")
    s5 = op([t], act("slice5", (B, H, W, 5)),
            f"r.slice({t},{{y}},{vec((B, H, W, C))},{vec((B, H, W, 5))},{{0,0,0,3}});", "slice5")
    op([s5, s3], act("concat_scalar", (B, H, W, C)), f"r.concat({s5},{s3},{{y}},{B * H * W},5,3);",
       "concat_scalar")
    # Batched matmul: computed x computed and computed x constant operands.
    xa = g.view(x, "x_batches", (B * C, H, W))
    bt = g.const("mm_b", init.xavier((B * C, W, 24), W, 24))
    op([xa, bt], act("matmul_const_b", (B * C, H, 24)),
       f"r.matmul({xa},{bt},{{y}},{B * C},{H},24,{W});", "matmul_const_b")
    xt = g.view(results[[r[0] for r in results].index("transpose_0132")][1], "xt_batches", (B * C, W, H))
    op([xa, xt], act("matmul_gram", (B * C, H, H)), f"r.matmul({xa},{xt},{{y}},{B * C},{H},{H},{W});",
       "matmul_gram")
    # Flatten and concatenate every result into the output vector.
    segments = [(name, g.tensors[y].shape) for name, y in results]
    cat, width = results[0][1], math.prod(g.tensors[results[0][1]].shape)
    for _, y in results[1:]:
        w = math.prod(g.tensors[y].shape)
        nxt = g.act("cat", (width + w,))
        g.op([cat, y], nxt, f"r.concat({cat},{y},{nxt},1,{width},{w});")
        cat, width = nxt, width + w
    assert width % B == 0
    out = g.view(cat, "zoo_out", (B, width // B))
    # Fill in the output ids of the recorded op strings.
    ops = []
    for ins, y, code in g.ops:
        ops.append((ins, y, code.replace("{y}", str(y))))
    g.ops = ops
    return g, out, segments


def load_spec(path: Path) -> dict:
    return json.loads(Path(path).read_text())
