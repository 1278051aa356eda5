"""The model.inc reader and the B200 packaging back end (ppocr_b200.package),
on CPU: every committed model.inc (fused and exporter-vocabulary) parses and
passes the checks, malformed files are rejected with the offending line,
and a package written from export.py-format shape directories has the
reference's layout (package.sh:9-51) with verified SHA-256 sums."""

import json
import shutil
import subprocess
from pathlib import Path

import pytest

from ppocr_b200 import models
from ppocr_b200 import package as P

MODELS = sorted(d for d in models.MODELS_SRC.iterdir() if (d / "model.inc").exists())


@pytest.mark.parametrize("d", MODELS, ids=lambda d: d.name)
def test_reader_parses_every_model(d):
    m = P.read_model_inc(d / "model.inc")
    P.validate(m)
    meta = json.loads((d / "meta.json").read_text())
    assert len(m.ops) == meta["operations"]
    assert list(m.input_shape) == meta["input_shape"]
    assert list(m.output_shape) == meta["output_shape"]
    assert m.constants["ARENA_ELEMENTS"] == meta["arena_elements"]
    assert m.constants["WEIGHT_ELEMENTS"] == meta["weight_elements"]
    assert m.constants["OUTPUT_ID"] == meta["output_id"]


def test_exporter_twins_do_the_same_work():
    """An `_xv` graph (export.py vocabulary) and its fused twin compute the
    same function: their contractions add up to the same flops."""
    for d in MODELS:
        twin = models.fused_twin(d.name)
        if not models.is_xv(d.name) or twin is None:
            continue
        a = P.read_model_inc(d / "model.inc")
        b = P.read_model_inc(models.MODELS_SRC / twin / "model.inc")
        assert sum(map(P.op_flops, a.ops)) == pytest.approx(sum(map(P.op_flops, b.ops)), rel=1e-12), d.name


def test_recognizer_flops_per_line():
    m = P.read_model_inc(models.MODELS_SRC / "rec_b512" / "model.inc")
    gflop_per_line = sum(map(P.op_flops, m.ops)) / 512 / 1e9
    # backbone 14.97 + neck 0.02 + 2048->120 0.02 (the CTC projection is the head's)
    assert gflop_per_line == pytest.approx(15.01, abs=0.01)


def _broken(tmp_path, edit):
    src = (models.MODELS_SRC / "rec_b2_xv" / "model.inc").read_text()
    f = tmp_path / "model.inc"
    f.write_text(edit(src))
    return f


@pytest.mark.parametrize("edit,message", [
    (lambda s: s.replace("r.softmax(", "r.softmax_v2(", 1), "unsupported operator `softmax_v2`"),
    (lambda s: s.replace("fused_pointwise_0<<<", "fused_pointwise_99<<<", 1), "undefined kernel"),
    (lambda s: s.replace("r.t.resize(132);", "r.t.resize(100);", 1), "outside the table"),
    (lambda s: s.replace("r.conv(12,13,15,", "r.conv(131,13,15,", 1), "before any op writes it"),
    (lambda s: s.replace("constexpr int OUTPUT_ID = 131;\n", "", 1), "missing constants"),
    (lambda s: s.replace("r.matmul(51,52,54,1,80,120,2048);", "r.matmul(51,52);", 1), "too few arguments"),
])
def test_reader_rejects(tmp_path, edit, message):
    f = _broken(tmp_path, edit)
    with pytest.raises(P.ModelIncError, match=message.replace("(", r"\(")) as exc:
        P.validate(P.read_model_inc(f))
    if "missing constants" not in message and "outside the table" not in message:
        assert ":" in str(exc.value).split("model.inc", 1)[1][:2], "the message names the line"


def test_reader_accepts_export_py_single_line_kernels(tmp_path):
    """export.py writes binary kernels on one line (export.py:956)."""
    src = (models.MODELS_SRC / "block_b16_xv" / "model.inc").read_text()
    one = ("__global__ void fused_binary_7(const Scalar* p0,const Scalar* p1,Scalar* y) "
           "{ int i=blockIdx.x*blockDim.x+threadIdx.x;if(i<8)y[i]=p0[i]+p1[i]; }\n")
    f = tmp_path / "model.inc"
    f.write_text(src.replace("constexpr size_t INPUT_ELEMENTS", one + "constexpr size_t INPUT_ELEMENTS", 1))
    m = P.read_model_inc(f)
    assert m.kernels["fused_binary_7"] == 3
    P.validate(m)


def _shape_dir(root: Path, name: str) -> Path:
    d = root / name
    d.mkdir(parents=True)
    shutil.copy2(models.MODELS_SRC / name / "model.inc", d / "model.inc")
    shutil.copy2(models.ensure_weights(name), d / "weights.f32")
    return d


def _abi_symbols(so: Path) -> set:
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}


def test_package_layout(tmp_path):
    """Shape directories in export.py's format -> package.sh's layout:
    models.tsv rows relative to the catalog, one shared weights.f32 per
    network, SHA256SUMS per shape, package.json over every file."""
    src = tmp_path / "src"
    rec = [_shape_dir(src / "rec", n) for n in ("rec_b2_xv", "rec_b64_xv")]
    det = [_shape_dir(src / "det", "det_b1_s128_xv")]
    out = P.package(tmp_path / "pkg", rec, det)
    P.verify(out)
    assert (out / "recognition" / "models.tsv").read_text().splitlines() == [
        "rec_b2_xv/model.so\tweights.f32", "rec_b64_xv/model.so\tweights.f32"]
    assert (out / "detection" / "models.tsv").read_text().splitlines() == ["det_b1_s128_xv/model.so\tweights.f32"]
    assert (out / "libppocr_b200.so").exists()
    for so in list(out.rglob("model.so")):
        syms = _abi_symbols(so)
        for s in ("ppocr_model_info", "ppocr_model_load_weights", "ppocr_model_create",
                  "ppocr_model_release_resources", "ppocr_model_enqueue", "ppocr_model_destroy",
                  "ppocr_model_error"):
            assert s in syms, (so, s)
    meta = json.loads((out / "package.json").read_text())
    assert meta["format_version"] == 1 and meta["model_abi_version"] == 2
    assert "recognition/weights.f32" in meta["files_sha256"]
    assert not any(k.endswith(("model.inc", "build.log")) for k in meta["files_sha256"])
    with pytest.raises(FileExistsError):
        P.package(out, rec, det)
    # a tampered file fails verification
    (out / "recognition" / "weights.f32").write_bytes(b"\0" * 64)
    with pytest.raises(ValueError, match="SHA-256"):
        P.verify(out)


def test_package_requires_shared_weights(tmp_path):
    src = tmp_path / "src"
    rec = [_shape_dir(src, "rec_b2"), _shape_dir(src, "rec_b2_xv")]  # fused vs exporter weight layouts
    with pytest.raises(ValueError, match="does not share the weights"):
        P.package(tmp_path / "pkg", rec, [])
    assert not (tmp_path / "pkg").exists(), "nothing is written before the checks pass"
