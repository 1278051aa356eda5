"""B200 back end of the reference's catalog packaging, and a reader for
exporter `model.inc` op lists.

The reference prepares a deployment in three steps
(tools/compiled_models/package.sh): export.py lowers an ONNX graph to one
`model.inc` + `weights.f32` per fixed shape; build.sh compiles
native/src/compiled/model_library.cu around each `model.inc` into
`model.so`; package.sh writes `models.tsv` per network (one row per shape,
library and weights paths relative to the catalog), keeps one verified copy
of the weights shared by every shape, a `SHA256SUMS` per shape and a
`package.json` with the SHA-256 of every file (package.sh:9-51).

This module is the B200 side of the last two steps. It takes shape
directories in export.py's output format -- from the reference's exporter
(any ONNX model it lowers) or from `ppocr_b200.modelgen` (the BASELINE
shapes: recognizer B = 64/256/512 at 48x320, detector 8 x 960^2) -- checks
every `model.inc` with the reader below, compiles it against this
repository's Runtime (`csrc/model_library.cu`, linked to libppocr_b200.so)
and writes the package in the reference's layout, so the reference's own
catalog engine (native/src/engine/model_engine_compiled.cpp:158-198) loads
it unchanged.

The reader (`read_model_inc`) parses the file export.py writes
(export.py:1032-1154): the size constants, the generated `__global__`
kernels, the tensor table (`r.t[i] = r.weights + o` / `r.arena + o`) and the
operator calls in graph order, each with its input and output tensor ids;
`validate` rejects what this Runtime cannot run (an unknown operator, an
undefined kernel, a tensor read before anything writes it, a table entry
out of range) with the line that caused it, as export.py rejects
unsupported ONNX operators; `op_flops` gives the multiply-add work of the
contractions.

ONNX lowering itself stays the reference's export.py: its `onnx` dependency
and the PP-OCRv6 ONNX files are not available offline here.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import re
import shutil
import subprocess
import sys
import tempfile
from dataclasses import dataclass, field
from pathlib import Path

from .build import ARCH, COMMON, CSRC, NVCC, build_library

# Runtime methods a model.inc may call (csrc/runtime.h), with the argument
# positions of their input tensor ids, of optional input ids (-1 = absent)
# and of the output id. upsample_concat_nhwc takes a list of inputs.
SIGNATURES = {
    "conv": ((0, 1), (12,), 2),
    "deconv": ((0, 1), (10,), 2),
    "gemm_epilogue": ((0, 1), (2, 3), 4),
    "matmul": ((0, 1), (), 2),
    "layernorm": ((0, 1, 2), (), 3),
    "softmax": ((0,), (), 1),
    "binary": ((0, 1), (), 2),
    "binary_fast": ((0, 1), (), 2),
    "unary": ((0,), (), 1),
    "transpose": ((0,), (), 1),
    "slice": ((0,), (), 1),
    "concat": ((0, 1), (), 2),
    "pad": ((0,), (), 1),
    "pad_nhwc": ((0,), (), 1),
    "pool": ((0,), (), 1),
    "pool_nhwc": ((0,), (), 1),
    "mean": ((0,), (), 1),
    "mean_nhwc": ((0,), (), 1),
    "resize_nearest": ((0,), (), 1),
    "resize_nearest_nhwc": ((0,), (), 1),
    # this Runtime's extensions (emitted by ppocr_b200.modelgen only)
    "attention": ((0,), (), 1),
    "resize_nearest_add_nhwc": ((0, 1), (), 2),
    "upsample_concat_nhwc": ((), (), 1),
}

CONSTANTS = ("INPUT_ELEMENTS", "OUTPUT_ELEMENTS", "OUTPUT_ID", "MODEL_INPUT_SHAPE", "MODEL_OUTPUT_RANK",
             "MODEL_OUTPUT_SHAPE", "ARENA_ELEMENTS", "WEIGHT_ELEMENTS")


class ModelIncError(ValueError):
    """A model.inc this Runtime cannot run; the message names the line."""


@dataclass
class Op:
    method: str               # Runtime method, or "kernel" for a generated kernel launch
    args: list                # parsed arguments (ints, floats, bools, nested lists)
    template: list            # template arguments (binary_fast<Op, AD, AM, BD, BM>)
    inputs: list              # tensor ids read
    output: int               # tensor id written
    line: int                 # 1-based line in model.inc
    kernel: str | None = None  # generated kernel name for "kernel" ops
    launch: tuple | None = None  # (grid, block, shared bytes) of a kernel launch


@dataclass
class ModelInc:
    path: Path
    constants: dict = field(default_factory=dict)
    kernels: dict = field(default_factory=dict)   # name -> parameter count
    n_tensors: int = 0
    tensors: dict = field(default_factory=dict)   # id -> ("weights" | "arena", element offset)
    ops: list = field(default_factory=list)

    @property
    def input_shape(self) -> tuple:
        return tuple(self.constants["MODEL_INPUT_SHAPE"])

    @property
    def output_shape(self) -> tuple:
        return tuple(self.constants["MODEL_OUTPUT_SHAPE"][: self.constants["MODEL_OUTPUT_RANK"]])

    def method_counts(self) -> dict:
        out: dict = {}
        for op in self.ops:
            out[op.method] = out.get(op.method, 0) + 1
        return out


# ---------------------------------------------------------------- parsing
def _split_top(s: str) -> list[str]:
    """Splits on commas outside braces and parentheses."""
    parts, depth, cur = [], 0, []
    for ch in s:
        if ch in "{(":
            depth += 1
        elif ch in "})":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append("".join(cur).strip())
            cur = []
        else:
            cur.append(ch)
    if cur or parts:
        parts.append("".join(cur).strip())
    return [p for p in parts if p != ""]


def _value(tok: str):
    tok = tok.strip()
    if tok.startswith("{"):
        if not tok.endswith("}"):
            raise ValueError(tok)
        return [_value(t) for t in _split_top(tok[1:-1])]
    if tok in ("true", "false"):
        return tok == "true"
    if re.fullmatch(r"[-+]?\d+", tok):
        return int(tok)
    f = tok[:-1] if tok.endswith(("f", "F")) else tok
    return float(f)


_CONST_RE = re.compile(r"constexpr\s+(?:size_t|int)\s+(\w+)(\[\d+\])?\s*=\s*([^;]+);")
_TABLE_RE = re.compile(r"r\.t\[(\d+)\]\s*=\s*r\.(weights|arena)\s*\+\s*(\d+)\s*;")
_RESIZE_RE = re.compile(r"r\.t\.resize\((\d+)\)\s*;")
_CALL_RE = re.compile(r"r\.(?:template\s+)?(\w+)(?:<([^>]*)>)?\((.*)\)\s*;\s*$")
_LAUNCH_RE = re.compile(r"r\.ops\.emplace_back\(\[&r\]\{\s*(\w+)<<<([^>]*)>>>\((.*)\)\s*;\s*\}\)\s*;\s*$")
_KERNEL_RE = re.compile(r"__global__\s+void\s+(\w+)\s*\(([^)]*)\)")


def read_model_inc(path: Path) -> ModelInc:
    """Parses a model.inc written in export.py's format."""
    path = Path(path)
    m = ModelInc(path=path)
    in_body = False
    for no, raw in enumerate(path.read_text().splitlines(), 1):
        line = raw.strip()
        if not line or line.startswith("//"):
            continue
        k = _KERNEL_RE.match(line)
        if k:
            params = [p for p in k.group(2).split(",") if p.strip()]
            m.kernels[k.group(1)] = len(params)
            continue
        c = _CONST_RE.match(line)
        if c and not in_body:
            try:
                m.constants[c.group(1)] = _value(c.group(3))
            except ValueError as exc:
                raise ModelIncError(f"{path}:{no}: cannot parse constant {c.group(1)}") from exc
            continue
        if c and c.group(1) == "WEIGHT_ELEMENTS":  # written after the body
            m.constants[c.group(1)] = _value(c.group(3))
            continue
        if line.startswith("template<class ModelRuntime> void build_model"):
            in_body = True
            continue
        if not in_body:
            continue
        if line == "}":
            in_body = False
            continue
        r = _RESIZE_RE.match(line)
        if r:
            m.n_tensors = int(r.group(1))
            continue
        t = _TABLE_RE.match(line)
        if t:
            m.tensors[int(t.group(1))] = (t.group(2), int(t.group(3)))
            continue
        launch = _LAUNCH_RE.match(line)
        if launch:
            ids = [int(x) for x in re.findall(r"r\.t\[(\d+)\]", launch.group(3))]
            if not ids:
                raise ModelIncError(f"{path}:{no}: kernel launch without tensors")
            cfg = [x.strip() for x in launch.group(2).split(",")]
            m.ops.append(Op("kernel", ids, [], ids[:-1], ids[-1], no, kernel=launch.group(1),
                            launch=tuple(cfg[:3])))
            continue
        call = _CALL_RE.match(line)
        if call:
            method = call.group(1)
            try:
                args = [_value(a) for a in _split_top(call.group(3))]
                tmpl = [_value(a) for a in _split_top(call.group(2))] if call.group(2) else []
            except ValueError as exc:
                raise ModelIncError(f"{path}:{no}: cannot parse the arguments of {method}") from exc
            if method not in SIGNATURES:
                raise ModelIncError(f"{path}:{no}: unsupported operator `{method}`")
            req, opt, out = SIGNATURES[method]
            if method == "upsample_concat_nhwc":
                ins = list(args[0])
            else:
                if len(args) <= max(req + (out,)):
                    raise ModelIncError(f"{path}:{no}: `{method}` has too few arguments")
                ins = [args[i] for i in req] + [args[i] for i in opt if i < len(args) and args[i] >= 0]
            m.ops.append(Op(method, args, tmpl, ins, args[out], no))
            continue
        raise ModelIncError(f"{path}:{no}: unrecognised statement: {line[:80]}")
    missing = [c for c in CONSTANTS if c not in m.constants]
    if missing:
        raise ModelIncError(f"{path}: missing constants {missing}")
    return m


# ------------------------------------------------------------- checking
def validate(m: ModelInc) -> None:
    """Raises ModelIncError for what this Runtime cannot run."""
    where = lambda op: f"{m.path}:{op.line}"  # noqa: E731
    n = m.n_tensors
    if n <= 0:
        raise ModelIncError(f"{m.path}: no tensor table (r.t.resize)")
    arena, weights = m.constants["ARENA_ELEMENTS"], m.constants["WEIGHT_ELEMENTS"]
    for i, (kind, off) in m.tensors.items():
        if not 0 <= i < n:
            raise ModelIncError(f"{m.path}: tensor {i} outside the table of {n}")
        limit = weights if kind == "weights" else arena
        if off > limit or (kind == "weights" and off == limit and limit > 0):
            raise ModelIncError(f"{m.path}: tensor {i} at {kind} offset {off} past {limit} elements")
    # Views (reshapes) share an arena offset with the tensor they alias.
    written_offsets = {m.tensors.get(0, ("arena", 0))[1]}
    written = {0}
    for op in m.ops:
        if op.method == "kernel":
            if op.kernel not in m.kernels:
                raise ModelIncError(f"{where(op)}: launch of undefined kernel `{op.kernel}`")
            if m.kernels[op.kernel] != len(op.args):
                raise ModelIncError(f"{where(op)}: `{op.kernel}` takes {m.kernels[op.kernel]} tensors, "
                                    f"launched with {len(op.args)}")
        for t in op.inputs + [op.output]:
            if not isinstance(t, int) or not 0 <= t < n or t not in m.tensors:
                raise ModelIncError(f"{where(op)}: `{op.method}` names tensor {t}, not in the table")
        for t in op.inputs:
            kind, off = m.tensors[t]
            if kind == "arena" and t not in written and off not in written_offsets:
                raise ModelIncError(f"{where(op)}: `{op.method}` reads tensor {t} before any op writes it")
        if m.tensors[op.output][0] == "weights":
            raise ModelIncError(f"{where(op)}: `{op.method}` writes into the weights")
        written.add(op.output)
        written_offsets.add(m.tensors[op.output][1])
    out = m.constants["OUTPUT_ID"]
    if out not in written and m.tensors.get(out, ("", -1))[1] not in written_offsets:
        raise ModelIncError(f"{m.path}: OUTPUT_ID {out} is never written")
    if math.prod(m.input_shape) != m.constants["INPUT_ELEMENTS"]:
        raise ModelIncError(f"{m.path}: INPUT_ELEMENTS disagrees with MODEL_INPUT_SHAPE")
    if math.prod(m.output_shape) != m.constants["OUTPUT_ELEMENTS"]:
        raise ModelIncError(f"{m.path}: OUTPUT_ELEMENTS disagrees with MODEL_OUTPUT_SHAPE")


def op_flops(op: Op) -> float:
    """Multiply-add work (2 flops each) of the contractions; 0 otherwise."""
    a = op.args
    if op.method == "conv":
        ws, ys = a[4], a[5]  # ws = {Co, Ci/groups, KH, KW}, ys = {N, Co, OH, OW}
        return 2.0 * math.prod(ys) * ws[1] * ws[2] * ws[3]
    if op.method == "deconv":
        xs, ws = a[3], a[4]  # ws = {Ci, Co, KH, KW}
        return 2.0 * math.prod(xs) * ws[1] * ws[2] * ws[3]
    if op.method == "gemm_epilogue":
        return 2.0 * a[5] * a[6] * a[7]
    if op.method == "matmul":
        return 2.0 * a[3] * a[4] * a[5] * a[6]
    if op.method == "attention":
        lines, seq, heads, dh = a[2], a[3], a[4], a[5]
        return 4.0 * lines * heads * seq * seq * dh
    return 0.0


def summary(m: ModelInc) -> dict:
    return {"path": str(m.path), "input_shape": list(m.input_shape), "output_shape": list(m.output_shape),
            "tensors": m.n_tensors, "operations": len(m.ops), "generated_kernels": len(m.kernels),
            "methods": m.method_counts(), "gflop": round(sum(op_flops(o) for o in m.ops) / 1e9, 3),
            "arena_bytes": 2 * m.constants["ARENA_ELEMENTS"], "weight_elements": m.constants["WEIGHT_ELEMENTS"]}


# ----------------------------------------------------------- packaging
def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 20), b""):
            h.update(block)
    return h.hexdigest()


def compile_shape(src_dir: Path, out_so: Path, detector: bool, lib_dir: Path) -> Path:
    """build.sh for this Runtime: csrc/model_library.cu around src_dir's
    model.inc, linked to libppocr_b200.so found two directories up at run
    time (the package root)."""
    out_so.parent.mkdir(parents=True, exist_ok=True)
    cmd = [NVCC, *ARCH, *COMMON, "-shared", "-I", str(src_dir), "-I", str(CSRC),
           f"-DPPOCR_MODEL_DETECTOR={1 if detector else 0}", str(CSRC / "model_library.cu"), "-o", str(out_so),
           "-L", str(lib_dir), "-lppocr_b200", "-Xlinker", "-rpath=$ORIGIN/../..",
           "-Xcompiler", "-fvisibility=hidden"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    (out_so.parent / "build.log").write_text(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"build of {src_dir} failed:\n{proc.stderr[-2000:]}")
    return out_so


def package(out: Path, recognition: list[Path] = (), detection: list[Path] = (),
            classifier: Path | None = None, jobs: int = 8) -> Path:
    """Writes a deployment package in package.sh's layout from shape
    directories in export.py's output format (model.inc + weights.f32; the
    directory name is the shape's name). Every model.inc is read and
    validated first; shapes of one network must share identical weights."""
    import concurrent.futures as cf

    out = Path(out)
    if (out / "package.json").exists():
        raise FileExistsError(f"{out}: use a fresh output directory; this package is already complete")
    groups = [("recognition", [Path(d) for d in recognition]), ("detection", [Path(d) for d in detection])]
    if not any(dirs for _, dirs in groups):
        raise ValueError("nothing to package")
    for kind, dirs in groups:
        for d in dirs:
            for f in ("model.inc", "weights.f32"):
                if not (d / f).exists():
                    raise FileNotFoundError(f"{d / f} missing (export.py writes model.inc and weights.f32)")
            validate(read_model_inc(d / "model.inc"))
        names = [d.name for d in dirs]
        if len(set(names)) != len(names):
            raise ValueError(f"{kind}: duplicate shape names {names}")
        if dirs:
            ref = dirs[0] / "weights.f32"
            for d in dirs[1:]:
                if _sha256(d / "weights.f32") != _sha256(ref):
                    raise ValueError(f"{kind}: {d.name} does not share the weights of {dirs[0].name}")
    lib = build_library()
    out.mkdir(parents=True, exist_ok=True)
    shutil.copy2(lib, out / "libppocr_b200.so")
    jobs_list = []
    for kind, dirs in groups:
        for d in dirs:
            jobs_list.append((d, out / kind / d.name / "model.so", kind == "detection"))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(lambda j: compile_shape(j[0], j[1], j[2], lib.parent), jobs_list))
    for kind, dirs in groups:
        if not dirs:
            continue
        root = out / kind
        shutil.copy2(dirs[0] / "weights.f32", root / "weights.f32")
        rows = []
        for d in dirs:
            shutil.copy2(d / "model.inc", root / d.name / "model.inc")
            rows.append(f"{d.name}/model.so\tweights.f32")
            (root / d.name / "SHA256SUMS").write_text(
                f"{_sha256(root / d.name / 'model.so')}  model.so\n{_sha256(root / 'weights.f32')}  ../weights.f32\n")
        (root / "models.tsv").write_text("\n".join(rows) + "\n")
    if classifier is not None:
        (out / "classifier").mkdir(exist_ok=True)
        for f in sorted(Path(classifier).iterdir()):
            if f.is_file():
                shutil.copy2(f, out / "classifier" / f.name)
    files = {}
    for p in sorted(out.rglob("*")):
        if p.is_file() and p.name not in ("package.json", "build.log", "export.log", "model.inc"):
            files[str(p.relative_to(out))] = _sha256(p)
    (out / "package.json").write_text(json.dumps({"format_version": 1, "model_abi_version": 2,
                                                  "files_sha256": files}, indent=2) + "\n")
    return out


def verify(out: Path) -> None:
    """Checks package.json and every SHA256SUMS against the files."""
    out = Path(out)
    meta = json.loads((out / "package.json").read_text())
    for rel, digest in meta["files_sha256"].items():
        if _sha256(out / rel) != digest:
            raise ValueError(f"{rel}: SHA-256 mismatch")
    for sums in out.rglob("SHA256SUMS"):
        for line in sums.read_text().splitlines():
            digest, name = line.split("  ", 1)
            if _sha256(sums.parent / name) != digest:
                raise ValueError(f"{sums.parent / name}: SHA-256 mismatch")


BENCHMARK_SHAPES = {"recognition": ["rec_b64", "rec_b256", "rec_b512"], "detection": ["det_b8"]}


def stage_benchmark_shapes(stage: Path, shapes: dict = BENCHMARK_SHAPES) -> dict:
    """Writes the BASELINE shapes in export.py's output format (model.inc +
    weights.f32 per shape directory) from ppocr_b200.modelgen."""
    from . import models

    dirs = {}
    for kind, names in shapes.items():
        dirs[kind] = []
        for name in names:
            d = Path(stage) / kind / name
            d.mkdir(parents=True, exist_ok=True)
            models.generate(name)
            shutil.copy2(models.MODELS_SRC / name / "model.inc", d / "model.inc")
            shutil.copy2(models.ensure_weights(name), d / "weights.f32")
            dirs[kind].append(d)
    return dirs


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("out", nargs="?", help="fresh output directory for the package")
    p.add_argument("--recognition", nargs="*", default=[], help="recognizer shape directories (export.py output)")
    p.add_argument("--detection", nargs="*", default=[], help="detector shape directories (export.py output)")
    p.add_argument("--classifier", help="classifier asset directory to copy")
    p.add_argument("--benchmark", action="store_true",
                   help="package the BASELINE shapes (recognizer B 64/256/512 at 48x320, detector 8 x 960^2)")
    p.add_argument("--read", nargs="*", default=[], help="read, validate and summarise model.inc files")
    a = p.parse_args(argv)
    if a.read:
        for f in a.read:
            m = read_model_inc(Path(f))
            validate(m)
            print(json.dumps(summary(m)))
        if not a.out:
            return 0
    if not a.out:
        p.error("an output directory is required")
    rec, det = [Path(d) for d in a.recognition], [Path(d) for d in a.detection]
    with tempfile.TemporaryDirectory() as tmp:
        if a.benchmark:
            dirs = stage_benchmark_shapes(Path(tmp))
            rec, det = rec + dirs["recognition"], det + dirs["detection"]
        out = package(Path(a.out), rec, det, Path(a.classifier) if a.classifier else None)
    verify(out)
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
