"""Catalog of the synthetic benchmark models and their compiled shapes.

Families share one weights file across shapes, like a reference catalog row
set sharing `weights.f32` (native/src/engine/model_engine_compiled.cpp:
186-190). Weights are generated deterministically on first use (seed below)
into lib/weights/, which is not committed.
"""

from __future__ import annotations

import json
from pathlib import Path

from . import modelgen
from .build import LIB_DIR, MODELS_SRC

SEED = 20261201
SPEC_DIR = MODELS_SRC / "specs"
WEIGHTS_DIR = LIB_DIR / "weights"

# name -> (family, batch, size) ; size is only used by the detector
SHAPES = {
    "rec_b512": ("recognizer", 512, None),
    "rec_b256": ("recognizer", 256, None),
    "rec_b64": ("recognizer", 64, None),
    "rec_b2": ("recognizer", 2, None),
    "det_b8": ("detector", 8, 960),
    "det_b1_s128": ("detector", 1, 128),
    "block_b16": ("block", 16, None),
    "block_b2": ("block", 2, None),
    "neck_b256": ("neck", 256, None),
    "neck_b4": ("neck", 4, None),
}


def spec(family: str) -> dict:
    return modelgen.load_spec(SPEC_DIR / f"{family}.json")


def graph(name: str):
    family, batch, size = SHAPES[name]
    s = spec(family)
    if family == "recognizer":
        return modelgen.build_recognizer(s, batch, SEED)
    if family == "block":
        return modelgen.build_block(s, batch, SEED)
    if family == "neck":
        return modelgen.build_neck(s, batch, SEED)
    return modelgen.build_detector(s, batch, size, SEED)


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
    return WEIGHTS_DIR / f"{SHAPES[name][0]}.f32"


def ensure_weights(name: str) -> Path:
    path = weights_path(name)
    g, _ = graph(name)
    consts, elements = g.weight_consts()
    if not path.exists() or path.stat().st_size != elements * 4:
        modelgen.write_weights(path, consts)
    return path


def library_path(name: str) -> Path:
    return LIB_DIR / "models" / name / f"model_{name}.so"


def write_catalog(family: str, names: list[str], directory: Path) -> Path:
    """A models.tsv catalog in the reference format (library, weights)."""
    directory.mkdir(parents=True, exist_ok=True)
    rows = []
    for n in names:
        rows.append(f"{library_path(n)}\t{weights_path(n)}")
    p = directory / "models.tsv"
    p.write_text("# library\tweights\n" + "\n".join(rows) + "\n")
    return p
