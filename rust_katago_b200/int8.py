"""Host-side mirror of the reference's INT8 projection API.

The reference's Rust types (crates/kata_nn/src/backends/int8.rs) map one to one:

================================  =====================================
reference (int8.rs)               here (C ABI underneath)
================================  =====================================
``QuantizedWeights::new`` :171    :func:`quantize_weights`
``Int8Weight::upload`` :222       :class:`Int8Weight`
``Int8Workspace::new``            :class:`Int8Workspace`
``project_half`` :1012            :meth:`Int8Workspace.project_half`
``project_residual`` :1052        :meth:`Int8Workspace.project_residual`
``ffn`` :1104                     :meth:`Int8Workspace.ffn`
``ffn_rms`` :1135                 :meth:`Int8Workspace.ffn_rms`
================================  =====================================

Device memory is passed as torch CUDA tensors (torch is only the allocator
here); every computation runs in ``libkatab200.so``.  Errors raise
:class:`rust_katago_b200._capi.KbError` carrying the library's message, the
equivalent of the reference's ``Err(String)``.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _capi
from ._capi import call, load


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        import torch

        return int(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def padded16(k: int) -> int:
    return (k + 15) // 16 * 16


def quantize_weights(w: np.ndarray):
    """CPU weight quantisation of the library (kb_int8_quantize_weights)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    q = np.zeros((n, padded16(k)), np.int8)
    s = np.zeros(n, np.float32)
    call("kb_int8_quantize_weights", w.ctypes.data, n, k, q.ctypes.data, s.ctypes.data)
    return q, s


class Int8Weight:
    """Quantised weight resident on the current device (Int8Weight::upload)."""

    def __init__(self, w: np.ndarray, layout: int = _capi.LAYOUT_PLAIN):
        w = np.ascontiguousarray(w, dtype=np.float32)
        n, k = w.shape
        h = ctypes.c_void_p()
        call("kb_int8_weight_upload", w.ctypes.data, n, k, layout, ctypes.byref(h))
        self._h = h
        vals = [ctypes.c_int() for _ in range(4)]
        qp, sp = ctypes.c_void_p(), ctypes.c_void_p()
        call("kb_int8_weight_info", h, *[ctypes.byref(v) for v in vals], ctypes.byref(qp), ctypes.byref(sp))
        self.n, self.k, self.kp, self.n_stored = (v.value for v in vals)
        self.q_ptr, self.scales_ptr = qp.value, sp.value
        self.layout = layout

    @property
    def handle(self):
        return self._h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().kb_int8_weight_destroy(h)
            except Exception:
                pass
            self._h = None


class Int8Workspace:
    """Per-stream INT8 scratch (Int8Workspace::new(rt, stream, rows, max_k, max_n))."""

    def __init__(self, rows: int, max_k: int, max_n: int, stream=None):
        self.stream = _stream(stream)
        h = ctypes.c_void_p()
        call("kb_int8_workspace_create", self.stream, rows, max_k, max_n, ctypes.byref(h))
        self._h = h
        q, s, hid = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        call("kb_int8_workspace_buffers", h, ctypes.byref(q), ctypes.byref(s), ctypes.byref(hid))
        self.quantized_ptr, self.scales_ptr, self.hidden_ptr = q.value, s.value, hid.value
        self.rows, self.max_k, self.max_n = rows, padded16(max_k), max_n

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().kb_int8_workspace_destroy(h)
            except Exception:
                pass
            self._h = None

    def project_half(self, input_f16, stride: int, weight: Int8Weight, output_f16, rows: int, stream=None):
        call("kb_int8_project_half", self._h, _stream(stream) if stream is not None else self.stream,
             _ptr(input_f16), stride, weight.handle, _ptr(output_f16), rows)

    def project_residual(self, input_f16, stride: int, weight: Int8Weight, residual_f32, rows: int, stream=None):
        call("kb_int8_project_residual", self._h, _stream(stream) if stream is not None else self.stream,
             _ptr(input_f16), stride, weight.handle, _ptr(residual_f32), rows)

    def ffn(self, input_f16, dual: Int8Weight, down: Int8Weight, output_f32, rows: int, stream=None):
        call("kb_int8_ffn", self._h, _stream(stream) if stream is not None else self.stream,
             _ptr(input_f16), dual.handle, down.handle, _ptr(output_f32), rows)

    def ffn_rms(self, gamma, eps: float, dual: Int8Weight, down: Int8Weight, residual_f32, rows: int, stream=None):
        call("kb_int8_ffn_rms", self._h, _stream(stream) if stream is not None else self.stream,
             _ptr(gamma), eps, dual.handle, down.handle, _ptr(residual_f32), rows)

    def ffn_gelu_rms(self, gamma, eps: float, up: Int8Weight, up_bias, down: Int8Weight, down_bias,
                     residual_bf16, rows: int, stream=None):
        call("kb_int8_ffn_gelu_rms", self._h, _stream(stream) if stream is not None else self.stream,
             _ptr(gamma), eps, up.handle, _ptr(up_bias), down.handle, _ptr(down_bias), _ptr(residual_bf16), rows)


def ffn_gelu_rms_noalloc(gamma, eps: float, up: Int8Weight, up_bias, down: Int8Weight, down_bias, residual_bf16,
                         rows: int, stream=None):
    """GELU FFN block without a workspace: scratch is a fixed static device
    array (at most ~900 tokens for C=768, F=3072); calls overlapping on the GPU race."""
    call("kb_int8_ffn_gelu_rms_noalloc", _stream(stream), _ptr(gamma), eps, up.handle, _ptr(up_bias), down.handle,
         _ptr(down_bias), _ptr(residual_bf16), rows)


def noalloc_prepare():
    """Look up the current device's no-alloc scratch address now (before a
    stream capture); the first ffn_gelu_rms_noalloc call does it otherwise."""
    call("kb_int8_noalloc_prepare")


# ------------------------------------------------------------------ kernel-level calls
def gemm_i32(a, w, dots, m: int, n: int, kp: int, stream=None):
    call("kb_int8_gemm_i32", _ptr(a), _ptr(w), _ptr(dots), m, n, kp, _stream(stream))


def linear(a, sa, w, sw, bias, m, n, kp, epilogue, out, ldo, act=0, out_dtype=_capi.DT_BF16,
           n_out=0, row_amax=None, stream=None):
    call("kb_int8_linear", _ptr(a), _ptr(sa), _ptr(w), _ptr(sw), _ptr(bias), m, n, kp, epilogue, act,
         out_dtype, _ptr(out), ldo, n_out, _ptr(row_amax), _stream(stream))


def quantize_rows(x, dtype, rows, width, stride, kp, q, scales, stream=None):
    call("kb_int8_quantize_rows", _ptr(x), dtype, rows, width, stride, kp, _ptr(q), _ptr(scales), _stream(stream))


def quantize_rows_amax(x, dtype, rows, width, stride, kp, row_amax, q, scales, stream=None):
    call("kb_int8_quantize_rows_amax", _ptr(x), dtype, rows, width, stride, kp, _ptr(row_amax), _ptr(q),
         _ptr(scales), _stream(stream))


def rms_quantize(x, dtype, rows, width, stride, gamma, eps, boundary_dtype, kp, q, scales, stream=None):
    call("kb_int8_rms_quantize", _ptr(x), dtype, rows, width, stride, _ptr(gamma), eps, boundary_dtype, kp,
         _ptr(q), _ptr(scales), _stream(stream))


def bf16_linear(a, w, bias, m, n, k, epilogue, out, ldo, act=0, out_dtype=_capi.DT_BF16, stream=None):
    call("kb_bf16_linear", _ptr(a), _ptr(w), _ptr(bias), m, n, k, epilogue, act, out_dtype, _ptr(out), ldo,
         _stream(stream))


def f16_linear(a, w, bias, m, n, k, epilogue, out, ldo, act=0, out_dtype=_capi.DT_F16, stream=None):
    """kb_f16_linear: binary16 operands, fp32 accumulation, the same epilogues."""
    call("kb_f16_linear", _ptr(a), _ptr(w), _ptr(bias), m, n, k, epilogue, act, out_dtype, _ptr(out), ldo,
         _stream(stream))
