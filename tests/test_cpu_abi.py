"""CPU tests of the C-ABI boundary: every symbol declared in include/*.h is
exported by the built libraries, PpocrModelInfo matches the reference
loader's checks, and host-side argument errors surface as messages. No
compute call needs a GPU here."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
INCLUDE = REPO / "include"


def declared(header: str) -> list[str]:
    text = (INCLUDE / header).read_text()
    text = re.sub(r"//.*", "", text)
    return re.findall(r"\b(ppocr_\w+)\s*\(", text)


def exported(so: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}


def test_library_exports_head_and_ops():
    from ppocr_b200 import capi

    syms = exported(capi.lib_path())
    for h in ("ppocr_b200_head.h", "ppocr_b200_ops.h"):
        names = declared(h)
        assert names, h
        missing = [n for n in names if n not in syms]
        assert not missing, f"{h}: {missing}"
    assert set(capi.SIGNATURES) <= syms


def test_model_libraries_export_abi():
    from ppocr_b200 import models

    names = declared("ppocr_b200_model_abi.h")
    assert len(names) == 11
    for n in models.SHAPES:
        syms = exported(models.library_path(n))
        missing = [s for s in names if s not in syms]
        assert not missing, f"{n}: {missing}"


@pytest.mark.parametrize("name", ["rec_b512", "rec_b2", "det_b8", "det_b1_s128"])
def test_model_info_passes_reference_loader_checks(name):
    """The validation of model_engine_compiled.cpp:51-66, restated."""
    from ppocr_b200 import capi, models

    lib = capi.ModelLibrary(models.library_path(name))
    info = lib.info
    meta = models.generate.__globals__["json"].loads((models.MODELS_SRC / name / "meta.json").read_text())
    assert info.abi_version == 2
    assert 1 <= info.output_rank <= 4
    assert info.output_element_bytes in (2, 4)
    assert all(v > 0 for v in info.input_shape)
    assert info.input_shape[1] == 3
    assert info.output_shape[0] == info.input_shape[0]
    assert info.weight_file_bytes == meta["weight_elements"] * 4
    assert info.scratch_bytes >= meta["arena_elements"] * 2
    assert (info.output_element_bytes == 4) == name.startswith("det")


def test_load_weights_rejects_wrong_size(tmp_path):
    from ppocr_b200 import capi, models

    lib = capi.ModelLibrary(models.library_path("rec_b2"))
    bad = tmp_path / "w.f32"
    bad.write_bytes(b"\0" * 16)
    with pytest.raises(capi.NativeError, match="Invalid compiled model weight size"):
        lib.load_weights(bad)
    with pytest.raises(capi.NativeError, match="Invalid compiled model weight size"):
        lib.load_weights(tmp_path / "missing.f32")


def test_create_rejects_small_scratch():
    from ppocr_b200 import capi, models

    lib = capi.ModelLibrary(models.library_path("rec_b2"))
    with pytest.raises(capi.NativeError, match="Invalid compiled model storage"):
        lib.create(0x1000, 0x2000, 16)
    with pytest.raises(capi.NativeError, match="Invalid compiled model storage"):
        lib.create(None, 0x2000, 1 << 40)


def test_enqueue_null_handle():
    from ppocr_b200 import capi, models

    lib = capi.ModelLibrary(models.library_path("rec_b2"))
    assert lib.dll.ppocr_model_enqueue(None, None, None, 1, None) == -1
    assert lib.error() == "Null model handle"


def test_op_entry_points_reject_bad_arguments():
    from ppocr_b200 import capi

    lib = capi.load()
    assert lib.ppocr_b200_gemm_epilogue(None, None, None, None, None, 4, 12, 8, 0, None) == -1
    assert b"invalid gemm_epilogue" in lib.ppocr_b200_last_error()
    assert lib.ppocr_b200_linear_argmax_prob(1, 1, 1, 1, 1, 1, 4, 120, 100, 512, 1, 1, 1, 1, None) == -1
    assert lib.ppocr_b200_last_error() == b"invalid WMMA classifier launch arguments"
    assert lib.ppocr_b200_ctc_collapse(None, None, -1, 40, 0, None, None, None, None) == -1
    nrb, nvb, cnt = ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    assert lib.ppocr_b200_classifier_workspace(1280, 18385, 16, 512, ctypes.byref(nrb), ctypes.byref(nvb),
                                               ctypes.byref(cnt)) == 0
    # The reference's shape (classifier.cu:520-536), not the B200 kernel's.
    assert (nrb.value, nvb.value, cnt.value) == (80, 36, 80 * 16 * 36)
    assert lib.ppocr_b200_classifier_workspace(1281, 18385, 8, 128, ctypes.byref(nrb), ctypes.byref(nvb),
                                               ctypes.byref(cnt)) == 0
    assert (nrb.value, nvb.value, cnt.value) == (161, 144, 161 * 144 * 8)


def test_reference_engine_loads_and_validates_catalog(tmp_path):
    """The reference's own catalog engine (native/src/engine/
    model_engine_compiled.cpp, unmodified, oracle/_ref/libref_engine.so) loads
    a catalog of this repository's libraries written by write_catalog (dlopen,
    dlsym of the seven symbols, PpocrModelInfo checks, profiles sorted by
    batch) and rejects a weights file of the wrong size with its own message.
    No CUDA call is made. Skipped where the reference tree was never present
    to build the engine."""
    engine = REPO / "oracle" / "_ref" / "libref_engine.so"
    if not engine.exists():
        pytest.skip("oracle/_ref/libref_engine.so not built (reference tree absent)")
    from ppocr_b200 import models

    lib = ctypes.CDLL(str(engine))
    lib.ref_engine_error.restype = ctypes.c_char_p
    lib.ref_engine_load.restype = ctypes.c_void_p
    lib.ref_engine_load.argtypes = [ctypes.c_char_p]
    lib.ref_engine_profiles.argtypes = [ctypes.c_void_p]
    lib.ref_engine_profile_shape.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_longlong)]
    lib.ref_engine_destroy.argtypes = [ctypes.c_void_p]
    for n in ("rec_b64", "rec_b2"):
        models.ensure_weights(n)
    catalog = models.write_catalog("recognizer", ["rec_b64", "rec_b2"], tmp_path / "ok")
    h = lib.ref_engine_load(str(catalog).encode())
    assert h, lib.ref_engine_error().decode()
    try:
        assert lib.ref_engine_profiles(h) == 2
        shapes = []
        for p in range(2):
            s = (ctypes.c_longlong * 4)()
            lib.ref_engine_profile_shape(h, p, s)
            shapes.append(tuple(s))
        assert shapes == [(2, 3, 48, 320), (64, 3, 48, 320)]
    finally:
        lib.ref_engine_destroy(h)
    bad = tmp_path / "w.f32"
    bad.write_bytes(b"\0" * 64)
    (tmp_path / "models.tsv").write_text(f"{models.library_path('rec_b2')}\t{bad}\n")
    assert not lib.ref_engine_load(str(tmp_path / "models.tsv").encode())
    assert b"Compiled weight size mismatch" in lib.ref_engine_error()
