"""Runs a generated graph (ppocr_b200.modelgen.Graph) on the CPU oracle.

Each recorded layer is executed with oracle/layers.py on the same FP16
weights the device receives (weights.f32 rounded to fp16, as
ppocr_model_load_weights packs them, model_library.cu:100-129 in the
reference). Test infrastructure only.
"""

from __future__ import annotations

import numpy as np
import torch

from . import layers as L


def _w(g, i):
    return L.rh(torch.from_numpy(np.ascontiguousarray(g.tensors[i].const)))


def run_graph(g, x_nchw: np.ndarray, output_id: int, capture: set | None = None):
    """x_nchw float32 [B,3,H,W] (the ABI input). Returns the output tensor as
    float32 in its stored layout and, optionally, intermediate tensors."""
    vals = {0: L.rh(torch.from_numpy(np.ascontiguousarray(x_nchw, dtype=np.float32)))}
    caps = {}

    def get(i):
        t = g.tensors[i]
        if t.alias_of is not None:
            return vals[t.alias_of].reshape(t.shape)
        return vals[i]

    for layer in g.layers:
        op = layer["op"]
        if op == "to_nhwc":
            y = get(layer["in"]).permute(0, 2, 3, 1).contiguous()
        elif op == "conv":
            x = get(layer["in"])
            w = _w(g, layer["w"])
            b = _w(g, layer["b"])
            y = L.conv_nhwc(x, w, b, layer["stride"], layer["pad"], layer["groups"], layer["act"])
        elif op == "gemm":
            res = get(layer["res"]) if layer["res"] >= 0 else None
            y = L.gemm(get(layer["in"]), _w(g, layer["w"]), _w(g, layer["b"]), res, layer["act"])
        elif op == "layernorm":
            y = L.layernorm(get(layer["in"]), _w(g, layer["scale"]), _w(g, layer["bias"]), layer["eps"])
        elif op == "attention":
            y = L.attention(get(layer["in"]), layer["heads"], layer["dh"], layer["scale"])
        elif op == "avgpool":
            y = L.pool_nhwc(get(layer["in"]), layer["k"], layer["s"], (0, 0), False)
        elif op == "resize_add":
            add = get(layer["add"])
            y = L.resize_nearest_nhwc(get(layer["in"]), add.shape[1], add.shape[2], *layer["scale"], addend=add)
        elif op == "resize":
            out_shape = g.tensors[layer["out"]].shape
            y = L.resize_nearest_nhwc(get(layer["in"]), out_shape[1], out_shape[2], *layer["scale"])
        elif op == "concat":
            y = torch.cat([get(layer["a"]), get(layer["b"])], dim=-1)
        elif op == "upsample_concat":
            # Runtime::upsample_concat_nhwc: each source nearest-resized to
            # the output size (resize_nhwc_kernel mapping), then concatenated.
            oh, ow = g.tensors[layer["out"]].shape[1:3]
            parts = []
            for i in layer["in"]:
                x = get(i)
                parts.append(L.resize_nearest_nhwc(x, oh, ow, np.float32(oh) / np.float32(x.shape[1]),
                                                   np.float32(ow) / np.float32(x.shape[2])))
            y = torch.cat(parts, dim=-1)
        elif op == "deconv":
            y = L.deconv_kxk(get(layer["in"]), _w(g, layer["w"]), _w(g, layer["b"]), layer["act"])
        else:
            raise ValueError(op)
        vals[layer["out"]] = y
        if capture and layer["out"] in capture:
            caps[layer["out"]] = y
    return get(output_id), caps
