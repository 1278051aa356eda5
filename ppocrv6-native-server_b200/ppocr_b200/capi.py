"""ctypes bindings of the C-ABI libraries (include/ppocr_b200_*.h).

This is the reference-side binding a host program would write (the
reference's Rust server binds its C ABI the same way through libloading,
server/src/native.rs:123-157). Loading fails loudly when the compiled
library is missing: there is no fallback path.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int, c_longlong, c_size_t, c_uint32, c_void_p
from pathlib import Path

from .build import LIB_DIR

_LIB = None


class NativeLibraryMissing(RuntimeError):
    pass


def lib_path() -> Path:
    return LIB_DIR / "libppocr_b200.so"


# (name, restype, argtypes) for every function in include/ppocr_b200_head.h,
# include/ppocr_b200_ops.h and include/ppocr_b200_preprocess.h.
V, I, F, S, L = c_void_p, c_int, c_float, c_size_t, c_longlong
PI, PF = POINTER(c_int), POINTER(c_float)
SIGNATURES = {
    "ppocr_b200_last_error": (c_char_p, []),
    "ppocr_b200_device_error": (I, []),
    "ppocr_b200_test_store_error_code": (I, [I, I]),
    "ppocr_b200_classifier_workspace": (I, [I, I, I, I, PI, PI, POINTER(c_size_t)]),
    "ppocr_b200_linear_argmax_prob": (I, [V, V, V, V, V, V, I, I, I, I, V, V, V, I, V]),
    "ppocr_b200_classifier_pack": (I, [V, V, I, I, V]),
    "ppocr_b200_classifier_run_packed": (I, [V, V, V, V, V, V, I, I, I, V, V, V, I, V]),
    "ppocr_b200_classifier_run_packed_noalloc": (I, [V, V, V, V, V, V, I, I, I, I, V]),

    "ppocr_b200_selected_class_vs_max_probability": (I, [V, V, V, V, V, I, I, I, I, V]),
    "ppocr_b200_logits_argmax_prob": (I, [V, I, I, V, V, V, I, V]),
    "ppocr_b200_ctc_collapse": (I, [V, V, I, I, I, V, V, V, V]),
    "ppocr_b200_conv_nhwc": (I, [V, V, V, V, I, I, I, I, I, I, I, I, I, I, I, I, I, V]),
    "ppocr_b200_stem_s2d_pack": (I, [V, V, I, I, V]),
    "ppocr_b200_stem_s2d_scratch_bytes": (S, [I, I, I]),
    "ppocr_b200_stem_conv_s2d": (I, [V, V, V, V, V, I, I, I, I, I, I, V]),
    "ppocr_b200_gemm_epilogue": (I, [V, V, V, V, V, I, I, I, I, V]),
    "ppocr_b200_matmul": (I, [V, V, V, I, I, I, I, V]),
    "ppocr_b200_layernorm": (I, [V, V, V, V, I, I, F, V]),
    "ppocr_b200_softmax": (I, [V, V, I, I, V]),
    "ppocr_b200_attention": (I, [V, V, I, I, I, I, F, V]),
    "ppocr_b200_pool_nhwc": (I, [V, V, I, I, I, I, I, I, I, I, I, I, I, V]),
    "ppocr_b200_pad_nhwc": (I, [V, V, I, I, I, I, I, I, I, I, V]),
    "ppocr_b200_resize_nearest_nhwc": (I, [V, V, V, I, I, I, I, I, I, F, F, V]),
    "ppocr_b200_concat": (I, [V, V, V, L, I, I, V]),
    "ppocr_b200_upsample_concat_nhwc": (I, [V, V, V, V, I, V, I, I, I, V]),
    "ppocr_b200_transpose": (I, [V, V, I, I, I, V]),
    "ppocr_b200_unary": (I, [V, V, L, I, F, F, V]),
    "ppocr_b200_binary_flat": (I, [V, V, V, L, I, I, I, I, I, V]),
    "ppocr_b200_mean_nhwc": (I, [V, V, I, I, I, V]),
    "ppocr_b200_deconv_nhwc": (I, [V, V, V, V, I, I, I, I, I, I, I, I, V]),
    "ppocr_b200_deconv_db_tail": (I, [V, V, V, I, V, V, I, V, I, I, I, I, V]),
    "ppocr_b200_binarize": (I, [V, V, S, F, V]),
    "ppocr_b200_dwpw_block": (I, [V, V, V, I, V, V, I, V, I, I, I, I, I, I, V]),
    "ppocr_b200_db_components_workspace": (S, [I, I, I, I]),
    "ppocr_b200_db_components": (I, [V, V, I, I, I, I, V, V, V, V, V, V]),
    "ppocr_b200_device_free": (I, [V]),
    "ppocr_b200_f32_to_f16": (I, [V, V, S, S, V]),
    "ppocr_b200_f16_to_f32": (I, [V, V, S, V]),
    # include/ppocr_b200_preprocess.h
    "ppocr_b200_resize_normalize_detector_padded": (I, [V, S, I, I, V, I, I, I, I, I, V]),
    "ppocr_b200_resize_normalize_detector": (I, [V, S, I, I, V, I, I, I, V]),
    "ppocr_b200_detector_preprocess": (I, [V, S, I, I, S, I, V, I, I, I, I, I, I, V]),
    "ppocr_b200_batch_roi_warp": (I, [V, S, I, I, V, V, V, I, I, I, I, V]),
    "ppocr_b200_roi_warp": (I, [V, S, I, I, V, V, V, I, I, I, I, I, V]),
    "ppocr_b200_line_tensors": (I, [V, V, V, V, V, I, I, V, I, V]),
}
PREP_F32_NCHW, PREP_F16_NHWC = 0, 1

MODEL_SIGNATURES = {
    "ppocr_model_info": (c_void_p, []),
    "ppocr_model_load_weights": (c_void_p, [c_char_p]),
    "ppocr_model_create": (c_void_p, [V, V, S, V]),
    "ppocr_model_release_resources": (None, [V]),
    "ppocr_model_enqueue": (I, [V, V, V, I, V]),
    "ppocr_model_destroy": (None, [V]),
    "ppocr_model_error": (c_char_p, []),
    "ppocr_model_enqueue_nhwc_f16": (I, [V, V, V, I, V]),
    "ppocr_model_op_count": (I, [V]),
    "ppocr_model_op_name": (c_char_p, [V, I]),
    "ppocr_model_profile_ops": (I, [V, V, I]),
}


def _bind(dll, table):
    for name, (res, args) in table.items():
        fn = getattr(dll, name)
        fn.restype = res
        fn.argtypes = args
    return dll


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        p = lib_path()
        if not p.exists():
            raise NativeLibraryMissing(f"{p} is not built; run __graft_entry__.build()")
        _LIB = _bind(ctypes.CDLL(str(p), mode=ctypes.RTLD_GLOBAL), SIGNATURES)
    return _LIB


class NativeError(RuntimeError):
    pass


def check(rc: int, lib=None) -> None:
    if rc != 0:
        lib = lib or load()
        raise NativeError(lib.ppocr_b200_last_error().decode())


class PpocrModelInfo(ctypes.Structure):
    """Layout of PpocrModelInfo (include/ppocr_b200_model_abi.h)."""

    _fields_ = [
        ("abi_version", c_uint32),
        ("input_shape", c_int * 4),
        ("output_rank", c_int),
        ("output_shape", c_int * 4),
        ("output_element_bytes", c_int),
        ("weight_file_bytes", c_size_t),
        ("scratch_bytes", c_size_t),
    ]


class PpocrModelResources(ctypes.Structure):
    _fields_ = [("blas", c_void_p)]


class ModelLibrary:
    """One dlopen'd model_<name>.so (Model ABI v2)."""

    def __init__(self, path: Path):
        load()  # the runtime library must be resident first
        if not Path(path).exists():
            raise NativeLibraryMissing(f"{path} is not built")
        self.path = Path(path)
        self.dll = _bind(ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL), MODEL_SIGNATURES)
        self.info = PpocrModelInfo.from_address(self.dll.ppocr_model_info())
        self.resources = PpocrModelResources()

    def error(self) -> str:
        return self.dll.ppocr_model_error().decode()

    def load_weights(self, path: Path) -> int:
        p = self.dll.ppocr_model_load_weights(str(path).encode())
        if not p:
            raise NativeError(self.error())
        return p

    def create(self, weights: int, scratch: int, scratch_bytes: int) -> int:
        h = self.dll.ppocr_model_create(weights, scratch, scratch_bytes, ctypes.byref(self.resources))
        if not h:
            raise NativeError(self.error())
        return h

    def enqueue(self, handle, inp: int, out: int, batch: int, stream: int) -> None:
        if self.dll.ppocr_model_enqueue(handle, inp, out, batch, stream) != 0:
            raise NativeError(self.error())

    def enqueue_nhwc_f16(self, handle, inp: int, out: int, batch: int, stream: int) -> None:
        if self.dll.ppocr_model_enqueue_nhwc_f16(handle, inp, out, batch, stream) != 0:
            raise NativeError(self.error())

    def destroy(self, handle) -> None:
        self.dll.ppocr_model_destroy(handle)

    def op_names(self, handle) -> list[str]:
        n = self.dll.ppocr_model_op_count(handle)
        return [self.dll.ppocr_model_op_name(handle, i).decode() for i in range(n)]

    def profile(self, handle) -> list[float]:
        n = self.dll.ppocr_model_op_count(handle)
        buf = (c_float * n)()
        if self.dll.ppocr_model_profile_ops(handle, buf, n) != 0:
            raise NativeError(self.error())
        return list(buf)
