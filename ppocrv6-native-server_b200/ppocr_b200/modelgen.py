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
"""

from __future__ import annotations

import json
import os
import math
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
            lines.append(code)
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


class Builder:
    """Emits layers into a Graph and records an oracle layer description."""

    def __init__(self, g: Graph, init: Init):
        self.g = g
        self.init = init
        self.n = 0

    def _name(self, kind):
        self.n += 1
        return f"{kind}_{self.n}"

    def to_nhwc(self, x):
        b, c, h, w = self.g.tensors[x].shape
        y = self.g.act("x_nhwc", (b, h, w, c))
        self.g.op([x], y, f"r.transpose({x},{y},{vec((b, c, h, w))},{vec((b, h, w, c))},{{0,2,3,1}});",
                  {"op": "to_nhwc", "in": x, "out": y})
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
        y = self.g.act(name, (b, oh, ow, co))
        self.g.op([x, wi, bi], y,
                  f"r.conv({x},{wi},{y},{vec((b, c, h, w))},{vec(wshape)},{vec((b, co, oh, ow))},"
                  f"{vec((ph, pw))},{vec(stride)},{{1,1}},{groups},true,true,{bi},{ACT[act]});",
                  {"op": "conv", "in": x, "w": wi, "b": bi, "out": y, "stride": list(stride),
                   "pad": [ph, pw], "groups": groups, "act": ACT[act]})
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
        y = self.g.act(name, (b, h, w, co))
        rows = b * h * w
        self.g.op([x, wi, bi], y, f"r.gemm_epilogue({x},{wi},{bi},-1,{y},{rows},{c},{co},{ACT[act]});",
                  {"op": "gemm", "in": x, "w": wi, "b": bi, "res": -1, "out": y, "act": ACT[act]})
        return y

    def linear(self, x, co, act="none", residual=-1, bias_std=0.01):
        shape = self.g.tensors[x].shape
        c = shape[-1]
        rows = math.prod(shape[:-1])
        name = self._name("linear")
        wi = self.g.const(name + "_w", self.init.xavier((co, c), c, co))
        bi = self.g.const(name + "_b", self.init.normal((co,), 0.0, bias_std))
        y = self.g.act(name, shape[:-1] + (co,))
        self.g.op([x, wi, bi] + ([residual] if residual >= 0 else []), y,
                  f"r.gemm_epilogue({x},{wi},{bi},{residual},{y},{rows},{c},{co},{ACT[act]});",
                  {"op": "gemm", "in": x, "w": wi, "b": bi, "res": residual, "out": y, "act": ACT[act]})
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
                  {"op": "layernorm", "in": x, "scale": si, "bias": bi, "out": y, "eps": eps})
        return y

    def attention(self, qkv, heads, head_dim):
        lines, seq, width = self.g.tensors[qkv].shape
        assert width == 3 * heads * head_dim
        scale = head_dim ** -0.5
        y = self.g.act(self._name("attn"), (lines, seq, heads * head_dim))
        self.g.op([qkv], y, f"r.attention({qkv},{y},{lines},{seq},{heads},{head_dim},{flit(scale)});",
                  {"op": "attention", "in": qkv, "out": y, "heads": heads, "dh": head_dim,
                   "scale": float(np.float32(scale))})
        return y

    def avgpool(self, x, k, s):
        b, h, w, c = self.g.tensors[x].shape
        oh, ow = (h - k[0]) // s[0] + 1, (w - k[1]) // s[1] + 1
        y = self.g.act(self._name("pool"), (b, oh, ow, c))
        self.g.op([x], y, f"r.pool_nhwc({x},{y},{vec((b, c, h, w))},{vec((b, c, oh, ow))},"
                          f"{vec(k)},{vec(s)},{{0,0}},false);",
                  {"op": "avgpool", "in": x, "out": y, "k": list(k), "s": list(s)})
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


def build_recognizer(spec: dict, batch: int, seed: int):
    """HGNet-style backbone + SVTR neck; output hidden [B, T, dim]."""
    height, width = spec["height"], spec["width"]
    g = Graph((batch, 3, height, width))
    bd = Builder(g, Init(seed))
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


def build_block(spec: dict, batch: int, seed: int):
    """Depthwise-separable NHWC block: dw KxK (+BN, act) -> 1x1 (+BN, act)."""
    g = Graph((batch, spec["channels"], spec["height"], spec["width"]))
    bd = Builder(g, Init(seed))
    x = bd.to_nhwc(0)
    c = spec["channels"]
    x = bd.conv_bn_act(x, c, spec["kernel"], act=spec["act"], depthwise=True)
    x = bd.pointwise(x, spec["out"], act=spec["act"])
    return g, x


def build_neck(spec: dict, batch: int, seed: int):
    """SVTR neck alone on [B, seq, dim] FP16 tokens (input viewed as
    [B, 1, seq, dim], where NCHW and NHWC coincide)."""
    seq, dim = spec["seq"], spec["dim"]
    g = Graph((batch, 1, seq, dim))
    bd = Builder(g, Init(seed))
    x = g.view(0, "tokens", (batch, seq, dim))
    for _ in range(spec["blocks"]):
        x = svtr_block(bd, x, spec["heads"], dim // spec["heads"], spec.get("mlp_ratio", 2))
    return g, x


def build_detector(spec: dict, batch: int, size: int, seed: int, fused_fpn_tail: bool = True):
    """Backbone at strides 2..32 + FPN(256) + DB head -> sigmoid map [B,1,S,S]."""
    g = Graph((batch, 3, size, size))
    bd = Builder(g, Init(seed))
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
        y = g.act(bd._name("fpn_add"), (b, h, w, c))
        sh, sw = h / hs, w / ws_
        g.op([td[i + 1], lat[i]], y,
             f"r.resize_nearest_add_nhwc({td[i + 1]},{lat[i]},{y},{vec((b, c, hs, ws_))},{vec((b, c, h, w))},"
             f"{flit(sh)},{flit(sw)});",
             {"op": "resize_add", "in": td[i + 1], "add": lat[i], "out": y, "scale": [sh, sw]})
        td[i] = y
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
                 {"op": "resize", "in": o, "out": y, "scale": [h0 / h, w0 / w]})
            ups.append(y)
        cat = ups[0]
        width = c0
        for u in ups[1:]:
            cu = g.tensors[u].shape[-1]
            y = g.act(bd._name("cat"), (b, h0, w0, width + cu))
            g.op([cat, u], y, f"r.concat({cat},{u},{y},{b * h0 * w0},{width},{cu});",
                 {"op": "concat", "a": cat, "b": u, "out": y})
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
        y = g.act(name, (b, 2 * h, 2 * w, co))
        g.op([x, wi, bi], y,
             f"r.deconv({x},{wi},{y},{vec((b, c, h, w))},{vec((c, co, 2, 2))},{vec((b, co, 2 * h, 2 * w))},"
             f"{{0,0}},{{2,2}},{{1,1}},true,{bi},{ACT[act]});",
             {"op": "deconv", "in": x, "w": wi, "b": bi, "out": y, "act": ACT[act]})
        x = y
    b, h, w, _ = g.tensors[x].shape
    out = g.view(x, "maps", (b, 1, h, w))
    return g, out


def load_spec(path: Path) -> dict:
    return json.loads(Path(path).read_text())
