"""Catalog of the synthetic benchmark models and their compiled shapes.

Families share one weights file across shapes, like a reference catalog row
set sharing `weights.f32` (native/src/engine/model_engine_compiled.cpp:
186-190). Weights are generated deterministically on first use (seed below)
into lib/weights/, which is not committed.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from . import modelgen
from .build import LIB_DIR, MODELS_SRC

SEED = 20261201
SPEC_DIR = MODELS_SRC / "specs"
WEIGHTS_DIR = LIB_DIR / "weights"

# name -> (family, batch, size) ; size is only used by the detector. Names
# ending in `_xv` are the exporter-vocabulary twins of a fused shape (same
# function, written only with what export.py emits; modelgen's module
# docstring): they compile against this repository's Runtime and, as test
# infrastructure, against the reference's own runtime (oracle/Makefile).
SHAPES = {
    "rec_b512": ("recognizer", 512, None),
    "rec_b256": ("recognizer", 256, None),
    "rec_b128": ("recognizer", 128, None),
    "rec_b64": ("recognizer", 64, None),
    "rec_b2": ("recognizer", 2, None),
    "det_b8": ("detector", 8, 960),
    "det_b1": ("detector", 1, 960),
    "det_b4": ("detector", 4, 960),
    "det_b1_s128": ("detector", 1, 128),
    "block_b16": ("block", 16, None),
    "block_b2": ("block", 2, None),
    "neck_b256": ("neck", 256, None),
    "neck_b4": ("neck", 4, None),
    "rec_b2_xv": ("recognizer", 2, None),
    "rec_b64_xv": ("recognizer", 64, None),
    "rec_b512_xv": ("recognizer", 512, None),
    "rec_b256_xv": ("recognizer", 256, None),
    "det_b1_s128_xv": ("detector", 1, 128),
    "det_b1_xv": ("detector", 1, 960),
    "det_b8_xv": ("detector", 8, 960),
    "block_b16_xv": ("block", 16, None),
    "neck_b256_xv": ("neck", 256, None),
    "zoo_xv": ("zoo", 2, None),
    # Runtime fusion test graphs: every fusable pair fused, or split back by
    # a later read of its intermediate (same chain output).
    "probe_fused": ("probe", 2, None),
    "probe_split": ("probe_split", 2, None),
}


def is_xv(name: str) -> bool:
    return name.endswith("_xv")


def fused_twin(name: str) -> str | None:
    """The fused shape computing the same function as an `_xv` shape."""
    base = name[:-3] if is_xv(name) else name
    return base if base in SHAPES else None


def spec(family: str) -> dict:
    return modelgen.load_spec(SPEC_DIR / f"{family}.json")


def graph(name: str):
    family, batch, size = SHAPES[name]
    xv = is_xv(name)
    if family == "zoo":
        g, out, _ = modelgen.build_zoo_xv(SEED)
        return g, out
    if family in ("probe", "probe_split"):
        return modelgen.build_fusion_probe(SEED, split=family == "probe_split", batch=batch)
    s = spec(family)
    if family == "recognizer":
        return modelgen.build_recognizer(s, batch, SEED, xv=xv)
    if family == "block":
        return modelgen.build_block(s, batch, SEED, xv=xv)
    if family == "neck":
        return modelgen.build_neck(s, batch, SEED, xv=xv)
    return modelgen.build_detector(s, batch, size, SEED, xv=xv)


def generate(name: str) -> dict:
    """Writes models/<name>/model.inc (+ meta.json); returns the metadata."""
    g, out = graph(name)
    family = SHAPES[name][0]
    meta = g.write(MODELS_SRC / name, out, detector=(family == "detector"))
    meta["family"] = family
    (MODELS_SRC / name / "meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    return meta


def generate_all() -> None:
    for name in SHAPES:
        generate(name)


def weights_path(name: str) -> Path:
    return WEIGHTS_DIR / f"{SHAPES[name][0]}{'_xv' if is_xv(name) else ''}.f32"


def ensure_weights(name: str) -> Path:
    path = weights_path(name)
    g, _ = graph(name)
    consts, elements = g.weight_consts()
    if not path.exists() or path.stat().st_size != elements * 4:
        modelgen.write_weights(path, consts)
    return path


def library_path(name: str) -> Path:
    return LIB_DIR / "models" / name / f"model_{name}.so"


def head_weights(hidden: int, vocab: int, seed: int = SEED, calibrated: bool = True):
    """The benchmark recognizer's CTC head as float32 (weight [hidden][vocab],
    bias [vocab]), the layout the reference loads (classifier.cu:611-659).

    W0, b0 are seeded Xavier / N(0, 0.01) draws. With calibrated=True and
    models/specs/recognizer_head.json present (written by
    tests/golden/make_head.py), the hidden-state direction every frame of the
    random-init recognizer shares is projected out of W0 and the result is
    scaled, and the blank class gets a bias, so that decoded lines hold many
    distinct tokens instead of one class repeated on every frame:
    W = gain * (I - u u^T) W0, b = b0 + blank_bias * e_blank."""
    init = modelgen.Init(seed + 1)
    w = init.xavier((hidden, vocab), hidden, vocab)
    b = init.normal((vocab,), 0.0, 0.01)
    path = SPEC_DIR / "recognizer_head.json"
    if calibrated and path.exists():
        head = json.loads(path.read_text())
        c = np.asarray(head["center"], np.float64)
        if c.size == hidden:
            u = c / np.linalg.norm(c)
            w64 = w.astype(np.float64)
            w = (head["gain"] * (w64 - np.outer(u, u @ w64))).astype(np.float32)
            b = b.copy()
            b[spec("recognizer")["blank"]] += np.float32(head["blank_bias"])
    return w, b


def write_catalog(family: str, names: list[str], directory: Path) -> Path:
    """A models.tsv catalog in the reference format (library, weights)."""
    directory.mkdir(parents=True, exist_ok=True)
    rows = []
    for n in names:
        rows.append(f"{library_path(n)}\t{weights_path(n)}")
    p = directory / "models.tsv"
    p.write_text("# library\tweights\n" + "\n".join(rows) + "\n")
    return p
