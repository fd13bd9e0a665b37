"""Host-side mirror of the reference's MXFP8 projection API.

Reference types (Rust_KataGo crates/kata_nn/src/backends/mxfp8.rs) and their
counterparts here (C ABI underneath, torch tensors only as device memory):

=====================================  ==========================================
reference (mxfp8.rs)                   here
=====================================  ==========================================
``dimensions`` :56                     :func:`dimensions`
``Mxfp8Kernels::quantize`` :209        :func:`quantize`
``Mxfp8Weight::upload_from_f32`` :290  :class:`Mxfp8Weight`
``Mxfp8Workspace::new`` :788           :class:`Mxfp8Workspace`
``begin_forward`` :977                 :meth:`Mxfp8Workspace.begin_forward`
``project_half`` / ``project_f32``     :meth:`Mxfp8Workspace.project`
``validate_completed_status`` :1181    :func:`validate_status`
=====================================  ==========================================
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _capi
from ._capi import call, load
from .int8 import _ptr, _stream

OUT_HALF, OUT_FLOAT, OUT_FLOAT_RESIDUAL, OUT_BF16, OUT_BF16_RESIDUAL = (
    _capi.MX_OUT_HALF, _capi.MX_OUT_FLOAT, _capi.MX_OUT_FLOAT_RESIDUAL, _capi.MX_OUT_BF16, _capi.MX_OUT_BF16_RESIDUAL)


def dimensions(rows: int, k: int):
    """(kp, blocks4, data_bytes, scale_bytes) of an MXFP8 operand."""
    kp, b4 = ctypes.c_int(), ctypes.c_int()
    db, sb = ctypes.c_size_t(), ctypes.c_size_t()
    call("kb_mxfp8_dimensions", rows, k, ctypes.byref(kp), ctypes.byref(b4), ctypes.byref(db), ctypes.byref(sb))
    return kp.value, b4.value, db.value, sb.value


def quantize(x, dtype: int, rows: int, k: int, stride: int, q, scales, status, layer: int = 0, stream=None):
    """Block-32 quantiser into caller buffers (q uint8 [rows*kp], scales uint8)."""
    call("kb_mxfp8_quantize", _ptr(x), dtype, rows, k, stride, _ptr(q), _ptr(scales), scales.numel(), _ptr(status),
         layer, _stream(stream))


def rms_quantize(x, dtype: int, rows: int, width: int, stride: int, gamma, eps: float, boundary_dtype: int, q,
                 scales, status, layer: int = 0, stream=None):
    """Fused RMSNorm -> 16-bit boundary -> MXFP8 into caller buffers."""
    call("kb_mxfp8_rms_quantize", _ptr(x), dtype, rows, width, stride, _ptr(gamma), eps, boundary_dtype, _ptr(q),
         _ptr(scales), scales.numel(), _ptr(status), layer, _stream(stream))


def reset_status(status, stream=None):
    call("kb_status_reset", _ptr(status), _stream(stream))


def validate_status(status) -> None:
    """Raises unless the downloaded status word is [0, 0xffffffff] (mxfp8.rs:1181-1200)."""
    flags, layer = int(status[0]), int(status[1])
    if flags == 0 and layer == _capi.NO_LAYER:
        return
    raise _capi.KbError(_capi.KB_E_NONFINITE,
                        f"MXFP8 forward rejected: flags={flags:#x} first_layer={layer} "
                        "(NaN=1 infinity=2 output_nonfinite=4 weight_overflow=8); discard all outputs")


class Mxfp8Weight:
    """Immutable MXFP8 weight on the current device, quantised from original fp32."""

    def __init__(self, w: np.ndarray, n: int | None = None, k: int | None = None, stride: int | None = None):
        w = np.ascontiguousarray(w, dtype=np.float32).ravel()
        if n is None:
            raise ValueError("n, k and stride are required for a flat weight")
        k = k if k is not None else stride
        stride = stride if stride is not None else k
        h = ctypes.c_void_p()
        call("kb_mxfp8_weight_upload", w.ctypes.data, n, k, stride, ctypes.byref(h))
        self._h = h
        vals = [ctypes.c_int() for _ in range(3)]
        qp, sp = ctypes.c_void_p(), ctypes.c_void_p()
        sb = ctypes.c_size_t()
        call("kb_mxfp8_weight_info", h, *[ctypes.byref(v) for v in vals], ctypes.byref(qp), ctypes.byref(sp),
             ctypes.byref(sb))
        self.n, self.k, self.kp = (v.value for v in vals)
        self.q_ptr, self.scales_ptr, self.scale_bytes = qp.value, sp.value, sb.value

    @property
    def handle(self):
        return self._h

    def download(self):
        """(q uint8 [n, kp], packed scales uint8) copied to the host."""
        q = np.zeros(self.n * self.kp, np.uint8)
        sc = np.zeros(self.scale_bytes, np.uint8)
        _copy_dtoh(q, self.q_ptr)
        _copy_dtoh(sc, self.scales_ptr)
        return q.reshape(self.n, self.kp), sc

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().kb_mxfp8_weight_destroy(h)
            except Exception:
                pass
            self._h = None


_cudart = None


def _copy_dtoh(host: np.ndarray, dev_ptr: int) -> None:
    """Synchronous device -> host copy of host.nbytes bytes through the CUDA
    runtime that torch ships (the same primary context as the library)."""
    global _cudart
    if _cudart is None:
        from pathlib import Path

        import nvidia.cuda_runtime

        lib = ctypes.CDLL(str(Path(nvidia.cuda_runtime.__path__[0]) / "lib" / "libcudart.so.12"))
        lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
        lib.cudaMemcpy.restype = ctypes.c_int
        _cudart = lib
    err = _cudart.cudaMemcpy(host.ctypes.data, dev_ptr, host.nbytes, 2)  # cudaMemcpyDeviceToHost
    if err != 0:
        raise RuntimeError(f"cudaMemcpy failed ({err})")


def gemm(a_q, a_scales, rows: int, w: Mxfp8Weight, out, ldo: int, out_kind: int, status, layer: int = 0,
         bias=None, act: int = _capi.ACT_NONE, stream=None):
    call("kb_mxfp8_gemm", _ptr(a_q), _ptr(a_scales), rows, w.handle, _ptr(bias), act, out_kind, _ptr(out), ldo,
         _ptr(status), layer, _stream(stream))


class Mxfp8Workspace:
    """Quantisation scratch for `rows` activations of up to `max_k` columns,
    bound to one stream, with its own sticky status word (Mxfp8Workspace::new)."""

    def __init__(self, rows: int, max_k: int, stream=None):
        import torch

        kp, _, data, scale = dimensions(rows, max_k)
        self.rows, self.max_k = rows, max_k
        self.q = torch.zeros(data, dtype=torch.uint8, device="cuda")
        self.scales = torch.zeros(scale, dtype=torch.uint8, device="cuda")
        self.status = torch.zeros(2, dtype=torch.int32, device="cuda")
        self.stream = _stream(stream)
        self.began = False

    def begin_forward(self):
        reset_status(self.status, self.stream)
        self.began = True

    def project(self, w: Mxfp8Weight, x, dtype: int, stride: int, out, out_kind: int, layer: int):
        """Quantise x [rows, stride] (16-bit) and run the block-scaled GEMM into out."""
        if not self.began:
            raise _capi.KbError(_capi.KB_E_STATE, "MXFP8 begin_forward must precede projections")
        if w.k > self.max_k:
            raise _capi.KbError(_capi.KB_E_INVALID, "projection K exceeds the workspace")
        call("kb_mxfp8_project", w.handle, _ptr(x), dtype, self.rows, stride, _ptr(self.q), _ptr(self.scales),
             self.scales.numel(), out_kind, _ptr(out), w.n, _ptr(self.status), layer, self.stream)

    def status_host(self):
        import torch

        torch.cuda.synchronize()
        return [int(v) & 0xFFFFFFFF for v in self.status.cpu().tolist()]
