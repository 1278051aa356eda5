"""Builds the sm_100a libraries of the B200 layer path with nvcc.

Outputs (git-ignored, but they travel with the source tree):
  lib/libppocr_b200.so                  runtime, kernels, head and op C-ABI
  lib/models/<name>/model_<name>.so     Model ABI v2 shell + generated graph

The model shells are compiled the way the reference compiles its catalog
(tools/compiled_models/build.sh:15-23: nvcc -shared model_library.cu with the
generated model.inc on the include path), here linked against
libppocr_b200.so instead of cuDNN/cuBLAS.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import subprocess
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent  # ppocrv6-native-server_b200/
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "lib"
MODELS_SRC = PKG_ROOT / "models"
REPO_ROOT = PKG_ROOT.parent

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-fvisibility=default", "--expt-relaxed-constexpr"]

LIB_SOURCES = ["common.cu", "tc_gemm.cu", "halo_conv.cu", "dwpw.cu", "stem_tc.cu", "spatial.cu", "seq.cu", "head.cu",
               "detect.cu", "components.cu", "preprocess.cu", "lines.cu", "runtime.cu", "capi.cu",
               "head_noalloc.cu", "attention_tc.cu", "matmul_tc.cu"]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + proc.stdout + proc.stderr)


def _stamp(paths: list[Path], extra: str = "") -> str:
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def _up_to_date(target: Path, stamp: str) -> bool:
    s = target.with_suffix(target.suffix + ".stamp")
    return target.exists() and s.exists() and s.read_text() == stamp


def _write_stamp(target: Path, stamp: str) -> None:
    target.with_suffix(target.suffix + ".stamp").write_text(stamp)


def build_library(force: bool = False, jobs: int = 8) -> Path:
    """Compiles csrc/*.cu into lib/libppocr_b200.so (incremental by content hash)."""
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    out = LIB_DIR / "libppocr_b200.so"
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((REPO_ROOT / "include").glob("*.h"))
    srcs = [CSRC / s for s in LIB_SOURCES]
    stamp = _stamp(srcs + headers, " ".join(ARCH + COMMON))
    if not force and _up_to_date(out, stamp):
        return out
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = obj_dir / (src.stem + ".o")
        _run([NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)])
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, srcs))
    _run([NVCC, *ARCH, "-shared", "-o", str(out), *map(str, objs)])
    _write_stamp(out, stamp)
    return out


def build_model(name: str, force: bool = False) -> Path:
    """Compiles the ABI shell around models/<name>/model.inc."""
    lib = build_library()
    src_dir = MODELS_SRC / name
    inc = src_dir / "model.inc"
    if not inc.exists():
        raise FileNotFoundError(inc)
    out_dir = LIB_DIR / "models" / name
    out_dir.mkdir(parents=True, exist_ok=True)
    out = out_dir / f"model_{name}.so"
    defines = []
    detector = (src_dir / "DETECTOR").exists()
    if detector:
        defines.append("-DPPOCR_MODEL_DETECTOR=1")
    stamp = _stamp([inc, CSRC / "model_library.cu", CSRC / "runtime.h", CSRC / "kernels.h",
                    REPO_ROOT / "include" / "ppocr_b200_model_abi.h"],
                   " ".join(ARCH + COMMON + defines) + str(lib.stat().st_mtime_ns))
    if not force and _up_to_date(out, stamp):
        return out
    _run([NVCC, *ARCH, *COMMON, *defines, "-shared", "-I", str(src_dir), "-I", str(CSRC),
          str(CSRC / "model_library.cu"), "-o", str(out),
          "-L", str(LIB_DIR), "-lppocr_b200", "-Xlinker", "-rpath=$ORIGIN/../..",
          "-Xcompiler", "-fvisibility=hidden"])
    _write_stamp(out, stamp)
    return out


def build_all(models: list[str] | None = None, jobs: int = 8) -> dict[str, Path]:
    build_library(jobs=jobs)
    names = models if models is not None else sorted(p.name for p in MODELS_SRC.iterdir() if (p / "model.inc").exists())
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        paths = list(ex.map(build_model, names))
    return dict(zip(names, paths))
