"""Seeded synthetic models and positions (no model file or dataset is shipped).

Distributions follow BASELINE config 3: every weight N(0, 0.02), RMSNorm and
trunk-tip gains 1 + N(0, 0.02), biases N(0, 0.02); positions have 22 binary
input planes with P(1) = 0.3 and 19 global features N(0, 1).  RoPE frequency
pairs are fixed per head (a direction per head times a geometric ladder of
magnitudes), standing in for the reference's learned 2-D RoPE frequencies.

The blob layout is the one documented for kb_model_blob_floats in
include/katab200.h; `blob_sections` lists it by name.  The nested topology
(the reference's TF3 graph) adds gate scales 1 + N(0, 0.02) and gate biases
N(0, 0.02) for its BN-gate-SiLU layers.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

STEM_K = 22 * 9 + 19


@dataclass(frozen=True)
class Topology:
    trunk_channels: int = 768
    num_blocks: int = 11
    num_heads: int = 12
    head_dim: int = 64
    ffn_channels: int = 3072
    precision: int = 0  # KB_PREC_INT8 (0) or KB_PREC_MXFP8 (1)
    # KB_PROJ_* per projection (qkv, out, ffn_up, ffn_down); 0 = follow `precision`
    proj_precision: tuple = (0, 0, 0, 0)
    int8_min_ffn_width: int = 0
    # KB_TOPO_FLAT (0) or KB_TOPO_NESTED (1: outer blocks of pairs_per_block
    # attention / SwiGLU FFN pairs at width mid_channels; ffn_channels is the
    # SwiGLU hidden width)
    topology: int = 0
    mid_channels: int = 0
    pairs_per_block: int = 0
    norm_eps: float = 0.0

    @property
    def nested(self) -> bool:
        return self.topology == 1

    def desc(self):
        from ._capi import ModelDesc

        return ModelDesc(self.trunk_channels, self.num_blocks, self.num_heads, self.head_dim, self.ffn_channels,
                         self.precision, (ctypes.c_int * 4)(*self.proj_precision), self.int8_min_ffn_width,
                         self.topology, self.mid_channels, self.pairs_per_block, self.norm_eps)

    def resolved_precision(self) -> tuple:
        """Each projection's precision as the model loader resolves it: "int8",
        "mxfp8" or "bf16" for (qkv, out, ffn_up, ffn_down); in the nested
        topology the unquantised 16-bit projections are "f16"."""
        names = {1: "int8", 2: "mxfp8", 3: "f16" if self.nested else "bf16"}
        base = 2 if self.precision == 1 else 1
        out = []
        for i, p in enumerate(self.proj_precision):
            p = p or base
            if i >= 2 and p == 1 and self.int8_min_ffn_width and self.ffn_channels < self.int8_min_ffn_width:
                p = 3
            out.append(names[p])
        return tuple(out)


B11C768 = Topology()
B11C768_MXFP8 = Topology(precision=1)
# The reference's TF3 b11c768 (native_model.rs:79-124): 11 outer blocks of 3
# attention / SwiGLU pairs at width 384, 12 heads x 32, SwiGLU hidden 1152.
TF3_B11C768 = Topology(768, 11, 12, 32, 1152, topology=1, mid_channels=384, pairs_per_block=3)
# Its FFN-scope INT8 recipe (the reference's default cudaint8backend scope,
# Int8Scope::Ffn): attention projections unquantised binary16.
TF3_B11C768_FFN = Topology(768, 11, 12, 32, 1152, topology=1, mid_channels=384, pairs_per_block=3,
                           proj_precision=(3, 3, 0, 0))


def blob_sections(t: Topology):
    """[(name, shape)] in blob order."""
    c, f, h, d = t.trunk_channels, t.ffn_channels, t.num_heads, t.head_dim
    secs = [("stem", (c, STEM_K))]
    if t.nested:
        m = t.mid_channels
        for i in range(t.num_blocks):
            secs += [(f"b{i}.pre_s", (c,)), (f"b{i}.pre_b", (c,)), (f"b{i}.pre_w", (m, c))]
            for j in range(t.pairs_per_block):
                p = f"b{i}.p{j}"
                secs += [(f"{p}.rms1", (m,)), (f"{p}.qkv", (3 * m, m)), (f"{p}.out", (m, m)),
                         (f"{p}.rope", (h, d // 2, 2)), (f"{p}.rms2", (m,)), (f"{p}.gate", (f, m)),
                         (f"{p}.up", (f, m)), (f"{p}.down", (m, f))]
            secs += [(f"b{i}.post_s", (m,)), (f"b{i}.post_b", (m,)), (f"b{i}.post_w", (c, m))]
        return secs + head_sections(c)
    for i in range(t.num_blocks):
        secs += [(f"b{i}.rms1", (c,)), (f"b{i}.qkv", (3 * c, c)), (f"b{i}.out", (c, c)), (f"b{i}.rms2", (c,)),
                 (f"b{i}.up", (f, c)), (f"b{i}.up_b", (f,)), (f"b{i}.down", (c, f)), (f"b{i}.down_b", (c,)),
                 (f"b{i}.rope", (h, d // 2, 2))]
    return secs + head_sections(c)


def head_sections(c):
    """Trunk tip and heads, shared by both topologies."""
    return [("tip_gamma", (c,)), ("tip_beta", (c,)),
            ("p1", (96, c)), ("g1", (96, c)), ("g1_b", (96,)), ("v1", (192, c)), ("v1_b", (192,)),
            ("g_matmul", (96, 288)), ("pass1", (96, 288)), ("pass1_b", (96,)), ("pass2", (6, 96)),
            ("bias2", (96,)), ("conv2p", (6, 96)), ("v2", (192, 576)), ("v2_b", (192,)),
            ("value", (3, 192)), ("value_b", (3,)), ("misc", (10, 192)), ("misc_b", (10,)),
            ("moremisc", (8, 192)), ("moremisc_b", (8,)), ("own", (192,))]


def blob_size(t: Topology) -> int:
    return int(sum(np.prod(s) for _, s in blob_sections(t)))


def split_blob(blob: np.ndarray, t: Topology) -> dict:
    out, off = {}, 0
    for name, shape in blob_sections(t):
        n = int(np.prod(shape))
        out[name] = blob[off:off + n].reshape(shape)
        off += n
    assert off == blob.size
    return out


def make_blob(t: Topology = B11C768, seed: int = 1234) -> np.ndarray:
    rng = np.random.default_rng(seed)
    parts = []
    for name, shape in blob_sections(t):
        leaf = name.split(".")[-1]
        if leaf in ("rms1", "rms2", "tip_gamma", "pre_s", "post_s"):
            a = 1.0 + 0.02 * rng.standard_normal(shape)
        elif leaf == "rope":
            h, pairs, _ = shape
            theta = rng.uniform(0, 2 * np.pi, size=(h, 1))
            mag = 0.8 * (1.0 / 1000.0) ** (np.arange(pairs) / max(1, pairs))[None, :]
            a = np.stack([mag * np.cos(theta), mag * np.sin(theta)], axis=-1)
        else:
            a = 0.02 * rng.standard_normal(shape)
        parts.append(np.asarray(a, np.float32).ravel())
    return np.concatenate(parts).astype(np.float32)


def make_positions(n: int, seed: int = 99):
    """(spatial [n, 22, 19, 19] in {0, 1}, global [n, 19] N(0,1)), fp32."""
    rng = np.random.default_rng(seed)
    spatial = (rng.random((n, 22, 19, 19)) < 0.3).astype(np.float32)
    glob = rng.standard_normal((n, 19)).astype(np.float32)
    return spatial, glob


def blob_floats_checked(t: Topology) -> int:
    """Blob size as the library computes it (must equal blob_size)."""
    from . import _capi

    count = ctypes.c_size_t()
    desc = t.desc()
    _capi.call("kb_model_blob_floats", ctypes.byref(desc), ctypes.byref(count))
    return int(count.value)
