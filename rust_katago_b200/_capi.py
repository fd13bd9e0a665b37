"""ctypes binding of ``libkatab200.so`` (the C ABI declared in include/katab200.h).

Loading fails loudly when the library has not been built: there is no
fallback implementation of any entry point.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkatab200.so"

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float
U = ctypes.c_uint64
PP = ctypes.POINTER(ctypes.c_void_p)
IP = ctypes.POINTER(ctypes.c_int)
STREAM = ctypes.c_size_t  # uintptr_t

# name -> (restype, argtypes); must list every function include/katab200.h declares.
SIGNATURES: dict[str, tuple] = {
    "kb_last_error": (ctypes.c_char_p, []),
    "kb_version": (I, []),
    "kb_device_check": (I, [I]),
    "kb_int8_quantize_weights": (I, [P, I, I, P, P]),
    "kb_int8_weight_upload": (I, [P, I, I, I, PP]),
    "kb_int8_weight_info": (I, [P, IP, IP, IP, IP, PP, PP]),
    "kb_int8_weight_destroy": (None, [P]),
    "kb_int8_gemm_i32": (I, [P, P, P, I, I, I, STREAM]),
    "kb_int8_linear": (I, [P, P, P, P, P, I, I, I, I, I, I, P, I, I, P, STREAM]),
    "kb_int8_quantize_rows": (I, [P, I, I, I, I, I, P, P, STREAM]),
    "kb_int8_quantize_rows_amax": (I, [P, I, I, I, I, I, P, P, P, STREAM]),
    "kb_int8_rms_quantize": (I, [P, I, I, I, I, P, F, I, I, P, P, STREAM]),
    "kb_int8_workspace_create": (I, [STREAM, I, I, I, PP]),
    "kb_int8_workspace_destroy": (None, [P]),
    "kb_int8_workspace_buffers": (I, [P, PP, PP, PP]),
    "kb_int8_project_half": (I, [P, STREAM, P, I, P, P, I]),
    "kb_int8_project_residual": (I, [P, STREAM, P, I, P, P, I]),
    "kb_int8_ffn": (I, [P, STREAM, P, P, P, P, I]),
    "kb_int8_ffn_rms": (I, [P, STREAM, P, F, P, P, P, I]),
    "kb_int8_ffn_gelu_rms": (I, [P, STREAM, P, F, P, P, P, P, P, I]),
    "kb_int8_ffn_gelu_rms_noalloc": (I, [STREAM, P, F, P, P, P, P, P, I]),
    "kb_int8_noalloc_prepare": (I, []),
    "kb_bf16_linear": (I, [P, P, P, I, I, I, I, I, I, P, I, STREAM]),
    "kb_f16_linear": (I, [P, P, P, I, I, I, I, I, I, P, I, STREAM]),
    "kb_attention": (I, [P, P, P, P, I, I, I, F, I, STREAM]),
    "kb_attention_amax": (I, [P, P, P, I, I, I, F, I, STREAM]),
    "kb_status_reset": (I, [P, STREAM]),
    "kb_mxfp8_dimensions": (I, [I, I, IP, IP, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "kb_mxfp8_quantize": (I, [P, I, I, I, I, P, P, ctypes.c_size_t, P, ctypes.c_uint32, STREAM]),
    "kb_mxfp8_rms_quantize": (I, [P, I, I, I, I, P, F, I, P, P, ctypes.c_size_t, P, ctypes.c_uint32, STREAM]),
    "kb_mxfp8_weight_upload": (I, [P, I, I, I, PP]),
    "kb_mxfp8_weight_info": (I, [P, IP, IP, IP, PP, PP, ctypes.POINTER(ctypes.c_size_t)]),
    "kb_mxfp8_weight_destroy": (None, [P]),
    "kb_mxfp8_gemm": (I, [P, P, I, P, P, I, I, P, ctypes.c_long, P, ctypes.c_uint32, STREAM]),
    "kb_mxfp8_project": (I, [P, P, I, I, I, P, P, ctypes.c_size_t, I, P, ctypes.c_long, P, ctypes.c_uint32, STREAM]),
    "kb_model_blob_floats": (I, [P, ctypes.POINTER(ctypes.c_size_t)]),
    "kb_model_load": (I, [P, P, ctypes.c_size_t, I, PP]),
    "kb_model_destroy": (None, [P]),
    "kb_model_file_parse": (I, [ctypes.c_char_p, P, P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), P]),
    "kb_model_load_file": (I, [ctypes.c_char_p, P, I, PP, P]),
    "kb_handle_create": (I, [P, I, I, PP]),
    "kb_handle_destroy": (None, [P]),
    "kb_handle_stream": (I, [P, ctypes.POINTER(ctypes.c_size_t)]),
    "kb_warmup": (I, [P, ctypes.POINTER(ctypes.c_int), I]),
    "kb_test_wait_timeout": (I, [ctypes.c_ulonglong, P, STREAM]),
    "kb_test_int8_gemm_i32_wait_limit": (I, [P, P, P, I, I, I, ctypes.c_ulonglong, P, STREAM]),
    "kb_submit": (I, [P, I, P, P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "kb_query": (I, [P, ctypes.c_uint64]),
    "kb_finish": (I, [P, ctypes.c_uint64, P, P, P, P, P, ctypes.POINTER(ctypes.c_uint32)]),
    "kb_forward_device": (I, [P, I, P, P, P, I]),
    "kb_read_status": (I, [P, ctypes.POINTER(ctypes.c_uint32)]),
    "kb_forward_trace": (I, [P, I, P, P, P, P]),
    "kb_decode_device": (I, [I, P, P, P, P, P, STREAM]),
    "kb_set_postprocess": (I, [P, P]),
    "kb_submit_rows": (I, [P, I, P, P, P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "kb_finish_rows": (I, [P, ctypes.c_uint64, P, P, P, P, P, ctypes.POINTER(ctypes.c_uint32)]),
}


class ModelDesc(ctypes.Structure):
    """kb_model_desc."""

    _fields_ = [("trunk_channels", ctypes.c_int), ("num_blocks", ctypes.c_int), ("num_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("ffn_channels", ctypes.c_int), ("precision", ctypes.c_int),
                ("proj_precision", ctypes.c_int * 4), ("int8_min_ffn_width", ctypes.c_int),
                ("topology", ctypes.c_int), ("mid_channels", ctypes.c_int), ("pairs_per_block", ctypes.c_int),
                ("norm_eps", ctypes.c_float)]

class PostProcessParams(ctypes.Structure):
    """kb_postprocess_params (ModelPostProcessParams, crates/kata_nn/src/desc.rs:671-695,
    and the model version); defaults are the reference's, version 17."""

    _fields_ = [("model_version", ctypes.c_int32), ("output_scale_multiplier", ctypes.c_float),
                ("td_score_multiplier", ctypes.c_double), ("score_mean_multiplier", ctypes.c_double),
                ("score_stdev_multiplier", ctypes.c_double), ("lead_multiplier", ctypes.c_double),
                ("variance_time_multiplier", ctypes.c_double), ("shortterm_value_error_multiplier", ctypes.c_double),
                ("shortterm_score_error_multiplier", ctypes.c_double)]

    DEFAULTS = dict(model_version=17, output_scale_multiplier=1.0, td_score_multiplier=20.0,
                    score_mean_multiplier=20.0, score_stdev_multiplier=20.0, lead_multiplier=20.0,
                    variance_time_multiplier=40.0, shortterm_value_error_multiplier=0.25,
                    shortterm_score_error_multiplier=30.0)

    @classmethod
    def make(cls, **kw) -> "PostProcessParams":
        unknown = set(kw) - set(cls.DEFAULTS)
        if unknown:
            raise TypeError(f"unknown post-processing parameters: {sorted(unknown)}")
        return cls(**dict(cls.DEFAULTS, **kw))


# Constants mirrored from include/katab200.h.
KB_OK, KB_E_INVALID, KB_E_CUDA, KB_E_STATE, KB_E_NONFINITE, KB_E_UNSUPPORTED = range(6)
PROJ_FOLLOW, PROJ_INT8, PROJ_MXFP8, PROJ_BF16 = range(4)
DT_F32, DT_F16, DT_BF16 = 0, 1, 2
EPI_I32, EPI_F16, EPI_RES_F32, EPI_16, EPI_RES16, EPI_SWIGLU16, EPI_F32 = range(7)
ACT_NONE, ACT_GELU, ACT_SILU = 0, 1, 2
LAYOUT_PLAIN, LAYOUT_SWIGLU_DUAL = 0, 1
PREC_INT8, PREC_MXFP8 = 0, 1
TOPO_FLAT, TOPO_NESTED = 0, 1
MX_OUT_HALF, MX_OUT_FLOAT, MX_OUT_FLOAT_RESIDUAL, MX_OUT_BF16, MX_OUT_BF16_RESIDUAL = range(5)
STATUS_NAN, STATUS_INF, STATUS_OUTPUT_NONFINITE, STATUS_WEIGHT_OVERFLOW = 1, 2, 4, 8
STATUS_UNSUPPORTED_ARCH, STATUS_TIMEOUT = 16, 32
NO_LAYER = 0xFFFFFFFF

_lib: ctypes.CDLL | None = None


class KbError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"katab200 error {code}: {message}")
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m rust_katago_b200.build` "
                "(there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(code: int) -> None:
    if code != KB_OK:
        msg = load().kb_last_error().decode(errors="replace")
        raise KbError(code, msg)


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
