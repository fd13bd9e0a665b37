"""Host mirror of the reference's NN evaluator boundary.

The reference's `Backend` trait (crates/kata_nn/src/backend.rs:206-410),
implemented by `CudaBackend` (src/backends/cuda.rs:2610-3105), maps to:

===========================================  ===========================================
reference                                    here (C ABI underneath)
===========================================  ===========================================
``load_model_file`` (cuda.rs:2618)           :meth:`CudaBackend.load_model`
``create_compute_handle`` (cuda.rs:2926)     :meth:`CudaBackend.create_compute_handle`
``warmup_batches``                           :meth:`ComputeHandle.warmup`
``submit_output`` (cuda.rs:2196)             :meth:`ComputeHandle.submit_output`
``query_output_done``                        :meth:`ComputeHandle.query_output_done`
``finish_output`` (cuda.rs:2510)             :meth:`ComputeHandle.finish_output`
``get_output``                               :meth:`ComputeHandle.get_output`
===========================================  ===========================================

Outputs are the raw heads (no final activation, backend.rs:279-280): policy
[n, 6, 362], value [n, 3], misc [n, 10], moremisc [n, 8], ownership [n, 361].
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _capi
from ._capi import call, load
from .synthetic import Topology

OUT_PER_POS = 6 * 362 + 3 + 10 + 8 + 361


@dataclass
class NNOutputs:
    policy: np.ndarray
    value: np.ndarray
    misc: np.ndarray
    moremisc: np.ndarray
    ownership: np.ndarray


def unpack_outputs(flat: np.ndarray, n: int) -> NNOutputs:
    """Split the packed device output [policy | value | misc | moremisc | ownership]."""
    o = 0
    pol = flat[o:o + n * 6 * 362].reshape(n, 6, 362)
    o += n * 6 * 362
    val = flat[o:o + n * 3].reshape(n, 3)
    o += n * 3
    misc = flat[o:o + n * 10].reshape(n, 10)
    o += n * 10
    more = flat[o:o + n * 8].reshape(n, 8)
    o += n * 8
    own = flat[o:o + n * 361].reshape(n, 361)
    return NNOutputs(pol, val, misc, more, own)


class Model:
    def __init__(self, topology: Topology, blob: np.ndarray, device: int = 0):
        blob = np.ascontiguousarray(blob, dtype=np.float32)
        self.topology = topology
        self.device = device
        desc = topology.desc()
        h = ctypes.c_void_p()
        call("kb_model_load", ctypes.byref(desc), blob.ctypes.data, blob.size, device, ctypes.byref(h))
        self._h = h

    @property
    def handle(self):
        return self._h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().kb_model_destroy(h)
            except Exception:
                pass
            self._h = None


class ComputeHandle:
    """One stream and workspace; not thread-safe (one thread per handle, backend.rs:102-104)."""

    def __init__(self, model: Model, max_batch: int, inputs_nhwc: bool = False):
        self.model = model
        self.max_batch = max_batch
        h = ctypes.c_void_p()
        call("kb_handle_create", model.handle, max_batch, 1 if inputs_nhwc else 0, ctypes.byref(h))
        self._h = h
        s = ctypes.c_size_t()
        call("kb_handle_stream", h, ctypes.byref(s))
        self.stream = int(s.value)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                load().kb_handle_destroy(h)
            except Exception:
                pass
            self._h = None

    def warmup(self, batches):
        arr = (ctypes.c_int * len(batches))(*batches)
        call("kb_warmup", self._h, arr, len(batches))

    def submit_output(self, spatial: np.ndarray, glob: np.ndarray, symmetry=None) -> int:
        """Enqueue n positions; `symmetry` ([n] ints in 0..7, or None for the
        identity) is each row's board symmetry, applied on the device as the
        input is gathered (the reference applies copy_inputs_with_symmetry on
        the host, cuda.rs:2234-2245).  Outputs come back in the network's frame,
        as the reference's raw heads do; decode_raw_outputs reverses them."""
        spatial = np.ascontiguousarray(spatial, dtype=np.float32)
        glob = np.ascontiguousarray(glob, dtype=np.float32)
        n = spatial.shape[0]
        sym_ptr = None
        if symmetry is not None:
            symmetry = np.ascontiguousarray(symmetry, dtype=np.int32)
            if symmetry.shape != (n,):
                raise ValueError("symmetry must hold one entry per position")
            sym_ptr = symmetry.ctypes.data
        tok = ctypes.c_uint64()
        call("kb_submit", self._h, n, spatial.ctypes.data, glob.ctypes.data, sym_ptr, ctypes.byref(tok))
        self._pending = getattr(self, "_pending", {})
        self._pending[tok.value] = n
        return tok.value

    def query_output_done(self, token: int) -> bool:
        r = load().kb_query(self._h, token)
        if r < 0:
            _capi.check(-r)
        return r == 1

    def finish_output(self, token: int) -> NNOutputs:
        n = self._pending.pop(token)
        out = NNOutputs(np.zeros((n, 6, 362), np.float32), np.zeros((n, 3), np.float32),
                        np.zeros((n, 10), np.float32), np.zeros((n, 8), np.float32), np.zeros((n, 361), np.float32))
        status = (ctypes.c_uint32 * 2)()
        call("kb_finish", self._h, token, out.policy.ctypes.data, out.value.ctypes.data, out.misc.ctypes.data,
             out.moremisc.ctypes.data, out.ownership.ctypes.data, status)
        return out

    def get_output(self, spatial: np.ndarray, glob: np.ndarray, symmetry=None) -> NNOutputs:
        return self.finish_output(self.submit_output(spatial, glob, symmetry))

    def forward_device(self, n: int, d_spatial, d_global, d_out, use_graph: bool = True):
        call("kb_forward_device", self._h, n, int(d_spatial.data_ptr()), int(d_global.data_ptr()),
             int(d_out.data_ptr()), 1 if use_graph else 0)

    def forward_trace(self, n: int, d_spatial, d_global, d_out, d_trace):
        """Device forward (no graph) that also records the stem output, every
        block's attention output and the final residual into d_trace."""
        call("kb_forward_trace", self._h, n, int(d_spatial.data_ptr()), int(d_global.data_ptr()),
             int(d_out.data_ptr()), int(d_trace.data_ptr()))

    def read_status(self):
        st = (ctypes.c_uint32 * 2)()
        call("kb_read_status", self._h, st)
        return int(st[0]), int(st[1])


class CudaBackend:
    """Factory mirroring the reference's backend object."""

    @staticmethod
    def load_model(topology: Topology, blob: np.ndarray, device: int = 0) -> Model:
        return Model(topology, blob, device)

    @staticmethod
    def create_compute_handle(model: Model, max_batch: int, inputs_nhwc: bool = False) -> ComputeHandle:
        return ComputeHandle(model, max_batch, inputs_nhwc)
