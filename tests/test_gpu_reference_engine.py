"""This repository's model libraries loaded through the reference's OWN
catalog engine (native/src/engine/model_engine_compiled.cpp, compiled
unmodified into oracle/_ref/libref_engine.so behind a C shim): a models.tsv
catalog written by ppocr_b200.models.write_catalog is parsed, every row
dlopen'd with its seven ABI symbols dlsym'd and its PpocrModelInfo validated
(model_engine_compiled.cpp:43-75, 160-198), weights shared per file, and
inference runs through Context::select_profile / set_input_shape /
bind_workspace / enqueue (76-156). The outputs must equal the ctypes path
bit for bit."""

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import rng

pytestmark = pytest.mark.gpu

ENGINE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_engine.so"


@pytest.fixture(scope="module")
def engine_lib():
    if not ENGINE.exists():
        pytest.fail(f"{ENGINE} is not built (make -C oracle ref)")
    lib = ctypes.CDLL(str(ENGINE))
    V, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.ref_engine_error.restype = ctypes.c_char_p
    lib.ref_engine_load.restype = V
    lib.ref_engine_load.argtypes = [ctypes.c_char_p]
    lib.ref_engine_profiles.argtypes = [V]
    lib.ref_engine_profile_shape.argtypes = [V, I, ctypes.POINTER(L)]
    lib.ref_engine_workspace_bytes.restype = L
    lib.ref_engine_workspace_bytes.argtypes = [V]
    lib.ref_engine_output_is_f32.argtypes = [V]
    lib.ref_engine_enqueue.argtypes = [V, I, I, V, V, V, L, V]
    lib.ref_engine_destroy.argtypes = [V]
    return lib


def _ours(name, x, cuda):
    from ppocr_b200 import pipeline

    m = pipeline.CompiledModel(name, cuda)
    try:
        out = m.output_tensor()
        stream = torch.cuda.Stream(cuda)
        m.enqueue_f32(torch.from_numpy(x).to(cuda), out, stream)
        stream.synchronize()
        return out[: x.shape[0]].cpu()
    finally:
        m.close()


@pytest.mark.parametrize("family,names,profile_name,batch", [
    ("recognizer", ["rec_b64", "rec_b2"], "rec_b2", 2),   # catalog order != profile order
    ("recognizer", ["rec_b64", "rec_b2"], "rec_b64", 37),  # partial batch of the larger shape
    ("detector", ["det_b1_s128"], "det_b1_s128", 1),
])
def test_catalog_through_reference_engine(native, cuda, engine_lib, tmp_path, family, names, profile_name, batch):
    from ppocr_b200 import capi, models

    for n in names:
        models.ensure_weights(n)
    catalog = models.write_catalog(family, names, tmp_path)
    h = engine_lib.ref_engine_load(str(catalog).encode())
    assert h, engine_lib.ref_engine_error().decode()
    try:
        # The engine sorts profiles by maximum batch.
        shapes = []
        for p in range(engine_lib.ref_engine_profiles(h)):
            s = (ctypes.c_longlong * 4)()
            engine_lib.ref_engine_profile_shape(h, p, s)
            shapes.append(tuple(s))
        assert [s[0] for s in shapes] == sorted(s[0] for s in shapes)
        lib = capi.ModelLibrary(models.library_path(profile_name))
        want_shape = tuple(lib.info.input_shape)
        profile = shapes.index(want_shape)
        x = rng(60 + batch).uniform(-1, 1, (batch,) + want_shape[1:]).astype(np.float32)
        dx = torch.from_numpy(x).to(cuda)
        out_shape = tuple(lib.info.output_shape[: lib.info.output_rank])
        f32 = engine_lib.ref_engine_output_is_f32(h)
        assert f32 == (family == "detector")
        out = torch.empty((batch,) + out_shape[1:], dtype=torch.float32 if f32 else torch.float16, device=cuda)
        ws = engine_lib.ref_engine_workspace_bytes(h)
        scratch = torch.empty(ws, dtype=torch.uint8, device=cuda)
        stream = torch.cuda.Stream(cuda)
        for _ in range(2):  # first enqueue (warm-up + capture), then a replay
            rc = engine_lib.ref_engine_enqueue(h, profile, batch, ctypes.c_void_p(dx.data_ptr()),
                                               ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(scratch.data_ptr()),
                                               ws, ctypes.c_void_p(stream.cuda_stream))
            assert rc == 0, engine_lib.ref_engine_error().decode()
            stream.synchronize()
            got = out.cpu()
            assert torch.equal(got, _ours(profile_name, x, cuda))
        assert native.ppocr_b200_device_error() == 0
    finally:
        engine_lib.ref_engine_destroy(h)



def test_package_through_reference_engine(native, cuda, engine_lib, tmp_path):
    """A deployment package written by ppocr_b200.package from shape
    directories in export.py's format (package.sh's layout: catalog rows
    relative to models.tsv, shared weights.f32, the runtime library at the
    package root) loads in the reference's engine and runs bit-identical to
    the ctypes path of the same shapes."""
    import shutil

    from ppocr_b200 import models
    from ppocr_b200 import package as P

    def shape_dir(name):
        d = tmp_path / "src" / name
        d.mkdir(parents=True)
        shutil.copy2(models.MODELS_SRC / name / "model.inc", d / "model.inc")
        shutil.copy2(models.ensure_weights(name), d / "weights.f32")
        return d

    out = P.package(tmp_path / "pkg", [shape_dir("rec_b2"), shape_dir("rec_b64")], [shape_dir("det_b1_s128")])
    P.verify(out)
    for kind, name, batch in (("recognition", "rec_b64", 5), ("detection", "det_b1_s128", 1)):
        h = engine_lib.ref_engine_load(str(out / kind / "models.tsv").encode())
        assert h, engine_lib.ref_engine_error().decode()
        try:
            shapes = []
            for p in range(engine_lib.ref_engine_profiles(h)):
                s = (ctypes.c_longlong * 4)()
                engine_lib.ref_engine_profile_shape(h, p, s)
                shapes.append(tuple(s))
            m = P.read_model_inc(out / kind / name / "model.inc")
            profile = shapes.index(tuple(m.input_shape))
            x = rng(90 + batch).uniform(-1, 1, (batch,) + tuple(m.input_shape[1:])).astype(np.float32)
            dx = torch.from_numpy(x).to(cuda)
            f32 = engine_lib.ref_engine_output_is_f32(h)
            out_t = torch.empty((batch,) + tuple(m.output_shape[1:]), dtype=torch.float32 if f32 else torch.float16,
                                device=cuda)
            ws = engine_lib.ref_engine_workspace_bytes(h)
            scratch = torch.empty(ws, dtype=torch.uint8, device=cuda)
            stream = torch.cuda.Stream(cuda)
            rc = engine_lib.ref_engine_enqueue(h, profile, batch, ctypes.c_void_p(dx.data_ptr()),
                                               ctypes.c_void_p(out_t.data_ptr()), ctypes.c_void_p(scratch.data_ptr()),
                                               ws, ctypes.c_void_p(stream.cuda_stream))
            assert rc == 0, engine_lib.ref_engine_error().decode()
            stream.synchronize()
            assert torch.equal(out_t.cpu(), _ours(name, x, cuda))
        finally:
            engine_lib.ref_engine_destroy(h)
