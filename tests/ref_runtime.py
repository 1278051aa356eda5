"""Binding of the reference's own compiled-model libraries (test oracle only).

oracle/_ref/models/<name>/model.so is the reference's
native/src/compiled/model_library.cu with runtime.cuh, spatial_kernels.cuh
and cutlass_gemm.cu compiled unmodified (cuDNN convolutions, cuBLAS /
cuBLASLt / CUTLASS GEMMs and the reference's own SIMT kernels) around the
exporter-vocabulary graph ppocrv6-native-server_b200/models/<name>/model.inc
(oracle/Makefile `ref-models`). It is bound here exactly as the reference's
catalog loader binds a model library: the seven Model ABI v2 symbols
(native/src/engine/model_engine_compiled.cpp:43-75), nothing else.
"""

from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_int, c_size_t, c_void_p
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[1]
REF_MODELS = REPO / "oracle" / "_ref" / "models"

_ABI = {
    "ppocr_model_info": (c_void_p, []),
    "ppocr_model_load_weights": (c_void_p, [c_char_p]),
    "ppocr_model_create": (c_void_p, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "ppocr_model_release_resources": (None, [c_void_p]),
    "ppocr_model_enqueue": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "ppocr_model_destroy": (None, [c_void_p]),
    "ppocr_model_error": (c_char_p, []),
}


def ref_model_path(name: str) -> Path:
    return REF_MODELS / name / "model.so"


class RefModel:
    """One reference model library: weights, scratch, handle (ABI v2)."""

    def __init__(self, name: str, device: torch.device):
        from ppocr_b200 import capi, models

        path = ref_model_path(name)
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle ref-models` where the "
                                    "reference tree is present")
        self.device = device
        self.dll = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        for sym, (res, args) in _ABI.items():
            fn = getattr(self.dll, sym)
            fn.restype, fn.argtypes = res, args
        self.info = capi.PpocrModelInfo.from_address(self.dll.ppocr_model_info())
        assert self.info.abi_version == 2
        self.resources = capi.PpocrModelResources()
        self.weights = self.dll.ppocr_model_load_weights(str(models.ensure_weights(name)).encode())
        if not self.weights:
            raise RuntimeError(self.error())
        self.scratch = torch.empty(self.info.scratch_bytes, dtype=torch.uint8, device=device)
        self.handle = self.dll.ppocr_model_create(self.weights, self.scratch.data_ptr(), self.info.scratch_bytes,
                                                  ctypes.byref(self.resources))
        if not self.handle:
            raise RuntimeError(self.error())
        self.output_shape = tuple(self.info.output_shape[: self.info.output_rank])
        self.output_dtype = torch.float16 if self.info.output_element_bytes == 2 else torch.float32

    def error(self) -> str:
        return self.dll.ppocr_model_error().decode()

    def run(self, x_nchw: np.ndarray) -> torch.Tensor:
        """Full-batch enqueue of f32 NCHW input; returns the output on the host."""
        x = torch.from_numpy(np.ascontiguousarray(x_nchw, dtype=np.float32)).to(self.device)
        out = torch.empty(self.output_shape, dtype=self.output_dtype, device=self.device)
        stream = torch.cuda.Stream(self.device)
        rc = self.dll.ppocr_model_enqueue(self.handle, x.data_ptr(), out.data_ptr(), x.shape[0],
                                          ctypes.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(self.error())
        stream.synchronize()
        return out.float().cpu()

    def close(self) -> None:
        from ppocr_b200 import capi

        if self.handle:
            self.dll.ppocr_model_destroy(self.handle)
            self.handle = None
        self.dll.ppocr_model_release_resources(ctypes.byref(self.resources))
        if self.weights:
            torch.cuda.synchronize(self.device)
            capi.load().ppocr_b200_device_free(ctypes.c_void_p(self.weights))
            self.weights = None
