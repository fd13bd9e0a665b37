"""Synthetic native KataGo v17 TF3 model files and the reference's lowering
of them — TEST INFRASTRUCTURE ONLY.

No model file of the reference's TF3 family ships with it, so the loader
(kb_model_file_parse) is tested by a round trip: `random_native` draws the
native layers of a model (its BN layers with means, variances, scales and
biases, its matrices in the file's in-first order, its convolutions in the
file's [Y, X, IC, OC] order), `write` serialises them as the reference's
parser reads them (crates/kata_nn/src/model_parser.rs: text tokens, weight
arrays as text or as "@BIN@" + little-endian fp32, optional gzip), and
`lower` restates independently what the reference does to them: the BN fold
in fp32 (model_parser.rs:273-287), the out-first transpose (native_model.rs:
375-388), the convolution re-order (model_parser.rs:219-234) and the head
channel remapping (native_model.rs:230-299, :430-455), in the blob order of
kb_model_blob_floats (include/katab200.h, KB_TOPO_NESTED).
"""

from __future__ import annotations

import gzip
import io

import numpy as np

BN_EPS = np.float32(2.0 ** -10)  # exactly representable: var = 1 - eps gives sqrt(var + eps) == 1


def _bn(rng, c, unit_scale=False):
    if unit_scale:
        # merged scale exactly 1 (the heads' BN must fold to unit scales)
        return dict(c=c, mean=np.zeros(c, np.float32), var=np.full(c, 1 - BN_EPS, np.float32),
                    scale=np.ones(c, np.float32), bias=(0.02 * rng.standard_normal(c)).astype(np.float32))
    return dict(c=c, mean=(0.05 * rng.standard_normal(c)).astype(np.float32),
                var=(1.0 + 0.2 * rng.random(c)).astype(np.float32),
                scale=(1.0 + 0.05 * rng.standard_normal(c)).astype(np.float32),
                bias=(0.02 * rng.standard_normal(c)).astype(np.float32))


def _w(rng, *shape):
    return (0.02 * rng.standard_normal(shape)).astype(np.float32)


def random_native(c=256, nb=2, pairs=2, mid=128, hidden=384, seed=0, policy_channels=2):
    """The native layers of a small TF3 model (in the file's own orders)."""
    rng = np.random.default_rng(seed)
    heads = mid // 32
    m = dict(c=c, nb=nb, pairs=pairs, mid=mid, hidden=hidden, heads=heads, pc=policy_channels,
             rms_eps=np.float32(1e-6),
             pp=[20.0, 20.0, 20.0, 20.0, 40.0, 0.25, 30.0],
             stem=_w(rng, 3, 3, 22, c), glob=_w(rng, 19, c), blocks=[])
    for _ in range(nb):
        b = dict(pre_bn=_bn(rng, c), pre_conv=_w(rng, 1, 1, c, mid), pairs=[], post_bn=_bn(rng, mid),
                 post_conv=_w(rng, 1, 1, mid, c))
        for _ in range(pairs):
            theta = rng.uniform(0, 2 * np.pi, size=(heads, 1))
            mag = 0.8 * (1.0 / 1000.0) ** (np.arange(16) / 16)[None, :]
            b["pairs"].append(dict(
                ln1=(1 + 0.02 * rng.standard_normal(mid)).astype(np.float32),
                q=_w(rng, mid, mid), k=_w(rng, mid, mid), v=_w(rng, mid, mid), o=_w(rng, mid, mid),
                freqs=np.stack([mag * np.cos(theta), mag * np.sin(theta)], axis=-1).astype(np.float32),
                ln2=(1 + 0.02 * rng.standard_normal(mid)).astype(np.float32),
                l1=_w(rng, mid, hidden), gate=_w(rng, mid, hidden), l2=_w(rng, hidden, mid)))
        m["blocks"].append(b)
    m["tip_bn"] = _bn(rng, c)
    m["p1"] = _w(rng, 1, 1, c, 96)
    m["g1"] = _w(rng, 1, 1, c, 96)
    m["g1_bn"] = _bn(rng, 96, unit_scale=True)
    m["gbias"] = _w(rng, 288, 96)
    m["p1_bn"] = _bn(rng, 96, unit_scale=True)
    m["p2"] = _w(rng, 1, 1, 96, policy_channels)
    m["pass1"] = _w(rng, 288, 96)
    m["pass1_b"] = _w(rng, 96)
    m["pass2"] = _w(rng, 96, policy_channels)
    m["v1"] = _w(rng, 1, 1, c, 192)
    m["v1_bn"] = _bn(rng, 192, unit_scale=True)
    m["v2"] = _w(rng, 576, 192)
    m["v2_b"] = _w(rng, 192)
    m["v3"] = _w(rng, 192, 3)
    m["v3_b"] = _w(rng, 3)
    m["sv3"] = _w(rng, 192, 6)
    m["sv3_b"] = _w(rng, 6)
    m["own"] = _w(rng, 1, 1, 192, 1)
    return m


class _Writer:
    def __init__(self, binary):
        self.binary = binary
        self.out = io.BytesIO()

    def line(self, *tokens):
        self.out.write((" ".join(str(t) for t in tokens) + "\n").encode())

    def floats(self, a):
        a = np.ascontiguousarray(a, np.float32).ravel()
        if self.binary:
            self.out.write(b"@BIN@")
            self.out.write(a.astype("<f4").tobytes())
            self.out.write(b"\n")
        else:
            self.line(*[repr(float(x)) for x in a])

    def conv(self, name, w):
        ky, kx, ic, oc = w.shape
        self.line(name, ky, kx, ic, oc, 1, 1)
        self.floats(w)

    def bn(self, name, b):
        self.line(name, b["c"], repr(float(BN_EPS)), 1, 1)
        for key in ("mean", "var", "scale", "bias"):
            self.floats(b[key])

    def act(self, name, kind="ACTIVATION_SILU"):
        self.line(name, kind)

    def mm(self, name, w):
        self.line(name, w.shape[0], w.shape[1])
        self.floats(w)

    def mb(self, name, b):
        self.line(name, b.size)
        self.floats(b)

    def rms(self, name, w, eps):
        self.line(name, w.size, repr(float(eps)))
        self.floats(w)


def serialise(m, binary=True, version=17, activation="ACTIVATION_SILU"):
    """The bytes of a native model file (uncompressed)."""
    w = _Writer(binary)
    c, mid = m["c"], m["mid"]
    w.line("tf3_test_model", version, 22, 19)
    w.line(*m["pp"])
    w.line(0, 0, 0, 0, 0, 0, 0, 0)  # metadata encoder, two preferences, five reserved
    w.line("trunk", m["nb"], c, mid, mid, 0, 0)
    w.line(0, 0, 0, 0, 0, 0)  # standard trunk-tip BN, five unused options
    w.conv("conv1", m["stem"])
    w.mm("ginputs", m["glob"])
    for i, b in enumerate(m["blocks"]):
        w.line("nested_bottleneck_block", f"block{i}", 2 * m["pairs"])
        w.bn(f"b{i}.prebn", b["pre_bn"])
        w.act(f"b{i}.preact", activation)
        w.conv(f"b{i}.preconv", b["pre_conv"])
        for j, p in enumerate(b["pairs"]):
            w.line("transformer_attention_block", f"b{i}.att{j}", m["heads"], m["heads"], 32, 32, 1, 1)
            w.rms(f"b{i}.att{j}.ln", p["ln1"], m["rms_eps"])
            for key in ("q", "k", "v", "o"):
                w.mm(f"b{i}.att{j}.{key}", p[key])
            w.line(f"b{i}.att{j}.rope", m["heads"], 16, 2)
            w.floats(p["freqs"])
            w.line("transformer_ffn_block", f"b{i}.ffn{j}", mid, m["hidden"], 1)
            w.rms(f"b{i}.ffn{j}.ln", p["ln2"], m["rms_eps"])
            w.mm(f"b{i}.ffn{j}.l1", p["l1"])
            w.mm(f"b{i}.ffn{j}.gate", p["gate"])
            w.mm(f"b{i}.ffn{j}.l2", p["l2"])
        w.bn(f"b{i}.postbn", b["post_bn"])
        w.act(f"b{i}.postact", activation)
        w.conv(f"b{i}.postconv", b["post_conv"])
    w.bn("trunktip", m["tip_bn"])
    w.act("trunktipact")
    w.line("policyhead", m["pc"])
    w.line(0, 0, 0)
    w.conv("p1", m["p1"])
    w.conv("g1", m["g1"])
    w.bn("g1bn", m["g1_bn"])
    w.act("g1act")
    w.mm("gpool2bias", m["gbias"])
    w.bn("p1bn", m["p1_bn"])
    w.act("p1act")
    w.conv("p2", m["p2"])
    w.mm("gpool2pass", m["pass1"])
    w.mb("gpool2passbias", m["pass1_b"])
    w.act("passact")
    w.mm("gpool2pass2", m["pass2"])
    w.line("valuehead")
    w.line(0, 0, 0)
    w.conv("v1", m["v1"])
    w.bn("v1bn", m["v1_bn"])
    w.act("v1act")
    w.mm("v2", m["v2"])
    w.mb("v2b", m["v2_b"])
    w.act("v2act")
    w.mm("v3", m["v3"])
    w.mb("v3b", m["v3_b"])
    w.mm("sv3", m["sv3"])
    w.mb("sv3b", m["sv3_b"])
    w.conv("vownership", m["own"])
    return w.out.getvalue()


def write(path, m, **kw):
    data = serialise(m, binary=str(path).endswith((".bin", ".bin.gz")), **kw)
    if str(path).endswith(".gz"):
        data = gzip.compress(data)
    with open(path, "wb") as f:
        f.write(data)


def fold(b):
    """merged_scale = scale / sqrt(var + eps), merged_bias = bias - merged_scale * mean, in fp32."""
    f = np.float32
    s = (b["scale"] / np.sqrt((b["var"] + BN_EPS).astype(f)).astype(f)).astype(f)
    return s, (b["bias"] - (s * b["mean"]).astype(f)).astype(f)


def _conv_of(w):
    """[Y, X, IC, OC] -> [OC, IC, Y, X]."""
    return np.ascontiguousarray(np.transpose(w, (3, 2, 0, 1)), np.float32)


def _remap(src, rows, mapping):
    out = np.zeros((rows,) + src.shape[1:], np.float32)
    for a, b in mapping:
        out[b] = src[a]
    return out


def lower(m):
    """(kb_model_desc shape fields, blob) of the reference's lowering."""
    parts = []
    stem = _conv_of(m["stem"]).reshape(m["c"], 198)
    parts.append(np.concatenate([stem, m["glob"].T], axis=1))
    for b in m["blocks"]:
        s, bias = fold(b["pre_bn"])
        parts += [s, bias, _conv_of(b["pre_conv"])]
        for p in b["pairs"]:
            parts += [p["ln1"], p["q"].T, p["k"].T, p["v"].T, p["o"].T, p["freqs"], p["ln2"], p["l1"].T,
                      p["gate"].T, p["l2"].T]
        s, bias = fold(b["post_bn"])
        parts += [s, bias, _conv_of(b["post_conv"])]
    s, bias = fold(m["tip_bn"])
    parts += [s, bias]
    parts += [_conv_of(m["p1"]), _conv_of(m["g1"]), fold(m["g1_bn"])[1], _conv_of(m["v1"]), fold(m["v1_bn"])[1],
              m["gbias"].T, m["pass1"].T, m["pass1_b"], _remap(m["pass2"].T, 6, [(0, 0), (1, 5)]),
              fold(m["p1_bn"])[1], _remap(_conv_of(m["p2"]).reshape(m["pc"], 96), 6, [(0, 0), (1, 5)]),
              m["v2"].T, m["v2_b"], m["v3"].T, m["v3_b"],
              _remap(m["sv3"].T, 10, [(0, 0), (1, 1), (2, 2), (3, 3)]),
              _remap(m["sv3_b"], 10, [(0, 0), (1, 1), (2, 2), (3, 3)]),
              _remap(m["sv3"].T, 8, [(4, 0), (5, 1)]), _remap(m["sv3_b"], 8, [(4, 0), (5, 1)]),
              _conv_of(m["own"]).reshape(192)]
    blob = np.concatenate([np.ascontiguousarray(p, np.float32).ravel() for p in parts])
    shape = dict(trunk_channels=m["c"], num_blocks=m["nb"], num_heads=m["heads"], head_dim=32,
                 ffn_channels=m["hidden"], mid_channels=m["mid"], pairs_per_block=m["pairs"],
                 norm_eps=float(m["rms_eps"]))
    return shape, blob
