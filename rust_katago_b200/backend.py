"""Host mirror of the reference's NN evaluator boundary.

The reference's `Backend` trait (crates/kata_nn/src/backend.rs:206-410),
implemented by `CudaBackend` (src/backends/cuda.rs:2610-3105), maps to:

===========================================  ===========================================
reference                                    here (C ABI underneath)
===========================================  ===========================================
``load_model_file`` (cuda.rs:2618)           :meth:`CudaBackend.load_model_file` (a native TF3
                                             file), :meth:`CudaBackend.load_model` (a blob)
``create_compute_handle`` (cuda.rs:2926)     :meth:`CudaBackend.create_compute_handle`
``warmup_batches``                           :meth:`ComputeHandle.warmup`
``submit_output`` (cuda.rs:2196)             :meth:`ComputeHandle.submit_output`
``query_output_done``                        :meth:`ComputeHandle.query_output_done`
``finish_output`` (cuda.rs:2510)             :meth:`ComputeHandle.finish_output`
``get_output``                               :meth:`ComputeHandle.get_output`
``decode_raw_outputs`` (output_postprocess   :meth:`ComputeHandle.submit_rows` /
.rs:29-112, in finish_output)                :meth:`ComputeHandle.finish_rows`, :func:`decode_device`
``postprocess_output`` (output_postprocess   the same, with a legal-move mask
.rs:140-330, eval.rs:675)
===========================================  ===========================================

``submit_output`` / ``finish_output`` return the raw heads (no final
activation, backend.rs:279-280): policy [n, 6, 362], value [n, 3], misc [n, 10],
moremisc [n, 8], ownership [n, 361].  ``submit_rows`` / ``finish_rows`` return
them decoded on the device (:class:`DecodedOutputs`).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _capi
from ._capi import call, load
from .synthetic import Topology

OUT_PER_POS = 6 * 362 + 3 + 10 + 8 + 361
DEC_PER_POS = 362 + 3 + 4 + 2 + 361

# kb_row_params: one row's decoding parameters (24 bytes, the C struct's layout).
ROW_PARAMS_DTYPE = np.dtype([("symmetry", "<i4"), ("policy_optimism", "<f4"), ("policy_temperature", "<f4"),
                             ("board_x", "<i4"), ("board_y", "<i4"), ("include_owner_map", "u1"),
                             ("next_player_white", "u1"), ("passing_hacks", "u1"), ("no_result_off", "u1")])
assert ROW_PARAMS_DTYPE.itemsize == 24


def row_params(n: int, symmetry=0, policy_optimism=0.0, policy_temperature=1.0, board_x=19, board_y=19,
               include_owner_map=1, next_player_white=1, passing_hacks=0, no_result_off=0) -> np.ndarray:
    """kb_row_params for n rows; each field a scalar or an [n] array.
    symmetry / policy_optimism / include_owner_map are NNResultBuf's fields
    (backend.rs); policy_temperature and passing_hacks MiscNNInputParams'
    nn_policy_temperature / enable_passing_hacks; no_result_off is
    ko_rule != Simple and scoring_rule != Territory (output_postprocess.rs:228)."""
    rows = np.zeros(n, ROW_PARAMS_DTYPE)
    for name, v in (("symmetry", symmetry), ("policy_optimism", policy_optimism),
                    ("policy_temperature", policy_temperature), ("board_x", board_x), ("board_y", board_y),
                    ("include_owner_map", include_owner_map), ("next_player_white", next_player_white),
                    ("passing_hacks", passing_hacks), ("no_result_off", no_result_off)):
        rows[name] = v
    return rows


@dataclass
class DecodedOutputs:
    """The NNOutput fields per row: policy [n, 362] (policy_probs), value [n, 3]
    (white win / loss / no-result), misc [n, 4] (score_mean, score_mean_sq,
    lead, var_time_left), moremisc [n, 2] (shortterm winloss / score error),
    ownership [n, 361] (white_owner_map; zeros where not requested)."""

    policy: np.ndarray
    value: np.ndarray
    misc: np.ndarray
    moremisc: np.ndarray
    ownership: np.ndarray


def unpack_decoded(flat: np.ndarray, n: int) -> DecodedOutputs:
    """Split the packed decoded output [policy | value | misc | moremisc | ownership]."""
    parts, o = [], 0
    for w in (362, 3, 4, 2, 361):
        parts.append(flat[o:o + n * w].reshape(n, w))
        o += n * w
    return DecodedOutputs(*parts)


def decode_device(n: int, d_raw, d_rows, d_legal, d_out, stream: int, **pp) -> None:
    """kb_decode_device on torch device tensors: d_raw the packed raw heads of
    n rows, d_rows n kb_row_params (uint8 [n, 24]), d_legal uint8 [n, 362] or
    None (decode only), d_out float32 [n * DEC_PER_POS]; keyword arguments
    override the post-processing defaults (_capi.PostProcessParams)."""
    params = _capi.PostProcessParams.make(**pp)
    call("kb_decode_device", n, int(d_raw.data_ptr()), int(d_rows.data_ptr()),
         None if d_legal is None else int(d_legal.data_ptr()), ctypes.byref(params), int(d_out.data_ptr()), stream)


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
    @classmethod
    def from_file(cls, path: str, recipe: Topology | None = None, device: int = 0) -> "Model":
        """kb_model_load_file: a native model file of the reference's TF3 family;
        the precision fields come from `recipe` (None = every projection INT8).
        The parsed shape is in .topology, the file's post-processing
        parameters in .postprocess."""
        self = cls.__new__(cls)
        desc = _capi.ModelDesc()
        count = ctypes.c_size_t()
        call("kb_model_file_parse", str(path).encode(), ctypes.byref(desc), None, 0, ctypes.byref(count), None)
        self.topology = Topology(desc.trunk_channels, desc.num_blocks, desc.num_heads, desc.head_dim,
                                 desc.ffn_channels, recipe.precision if recipe else 0,
                                 tuple(recipe.proj_precision) if recipe else (0, 0, 0, 0),
                                 recipe.int8_min_ffn_width if recipe else 0, desc.topology, desc.mid_channels,
                                 desc.pairs_per_block, float(desc.norm_eps))
        self.device = device
        self.postprocess = _capi.PostProcessParams()
        h = ctypes.c_void_p()
        rdesc = recipe.desc() if recipe else None
        call("kb_model_load_file", str(path).encode(), ctypes.byref(rdesc) if rdesc else None, device,
             ctypes.byref(h), ctypes.byref(self.postprocess))
        self._h = h
        return self

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

    def set_postprocess(self, **pp) -> None:
        """Post-processing parameters for submit_rows (ModelPostProcessParams and
        the model version; unspecified fields keep the reference defaults)."""
        params = _capi.PostProcessParams.make(**pp)
        call("kb_set_postprocess", self._h, ctypes.byref(params))

    def submit_rows(self, spatial: np.ndarray, glob: np.ndarray, rows: np.ndarray, legal=None) -> int:
        """Enqueue n positions evaluated under rows['symmetry'] and decoded on
        the device (decode_raw_outputs); with legal ([n, 362] booleans, pass
        last) post-processed too (postprocess_output)."""
        spatial = np.ascontiguousarray(spatial, dtype=np.float32)
        glob = np.ascontiguousarray(glob, dtype=np.float32)
        n = spatial.shape[0]
        rows = np.ascontiguousarray(rows, dtype=ROW_PARAMS_DTYPE)
        if rows.shape != (n,):
            raise ValueError("rows must hold one kb_row_params per position")
        legal_ptr = None
        if legal is not None:
            legal = np.ascontiguousarray(legal, dtype=np.uint8)
            if legal.shape != (n, 362):
                raise ValueError("legal must be [n, 362]")
            legal_ptr = legal.ctypes.data
        tok = ctypes.c_uint64()
        call("kb_submit_rows", self._h, n, spatial.ctypes.data, glob.ctypes.data, rows.ctypes.data, legal_ptr,
             ctypes.byref(tok))
        self._pending = getattr(self, "_pending", {})
        self._pending[tok.value] = n
        return tok.value

    def finish_rows(self, token: int) -> DecodedOutputs:
        n = self._pending.pop(token)
        out = DecodedOutputs(np.zeros((n, 362), np.float32), np.zeros((n, 3), np.float32),
                             np.zeros((n, 4), np.float32), np.zeros((n, 2), np.float32),
                             np.zeros((n, 361), np.float32))
        status = (ctypes.c_uint32 * 2)()
        call("kb_finish_rows", self._h, token, out.policy.ctypes.data, out.value.ctypes.data, out.misc.ctypes.data,
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
    def load_model_file(path: str, recipe: Topology | None = None, device: int = 0) -> Model:
        """Backend::load_model_file (backend.rs:206-410) for the TF3 family."""
        return Model.from_file(path, recipe, device)

    @staticmethod
    def create_compute_handle(model: Model, max_batch: int, inputs_nhwc: bool = False) -> ComputeHandle:
        return ComputeHandle(model, max_batch, inputs_nhwc)
