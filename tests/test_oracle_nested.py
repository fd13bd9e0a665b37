"""CPU checks of the nested (TF3) topology's host side: the descriptor's
validation in the library (kb_model_blob_floats needs no GPU), the blob layout
shared by the synthetic generator, the library and the oracle's parser, and
the oracle's gate and attention-scale definitions."""

import ctypes

import numpy as np
import pytest

import oracle
import oracle.trunk_nested as onest
from rust_katago_b200 import _capi, synthetic

TF3 = synthetic.TF3_B11C768


def blob_floats(t):
    return synthetic.blob_floats_checked(t)


def test_blob_layout_agrees():
    for t in (TF3, synthetic.TF3_B11C768_FFN, synthetic.Topology(256, 2, 4, 32, 384, topology=1, mid_channels=128,
                                                                 pairs_per_block=2)):
        n = synthetic.blob_size(t)
        assert blob_floats(t) == n
        blob = synthetic.make_blob(t, 3)
        w = onest.parse(blob, (t.trunk_channels, t.num_blocks, t.pairs_per_block, t.num_heads, t.mid_channels,
                                t.ffn_channels))
        parts = synthetic.split_blob(blob, t)
        assert np.array_equal(w["0.0.gate"], parts["b0.p0.gate"])
        assert np.array_equal(w["tip_g"], parts["tip_gamma"])


@pytest.mark.parametrize("kw,msg", [
    (dict(head_dim=64, num_heads=6), "head_dim 32"),
    (dict(mid_channels=768), "mid < C"),
    (dict(ffn_channels=3 * 384 + 8), "3\\*mid"),
    (dict(pairs_per_block=0), "pairs"),
    (dict(precision=1), "KB_PREC_INT8"),
    (dict(proj_precision=(0, 0, 3, 0)), "FFN INT8"),
    (dict(int8_min_ffn_width=2048), "unquantised"),
])
def test_descriptor_validation(kw, msg):
    base = dict(trunk_channels=768, num_blocks=11, num_heads=12, head_dim=32, ffn_channels=1152, topology=1,
                mid_channels=384, pairs_per_block=3)
    base.update(kw)
    with pytest.raises(_capi.KbError, match=msg):
        blob_floats(synthetic.Topology(**base))


def test_flat_descriptor_rejects_unknown_topology():
    with pytest.raises(_capi.KbError, match="topology"):
        blob_floats(synthetic.Topology(topology=7))


def test_gate_and_scale_definitions():
    x = np.array([[-3.0, 0.25, 1.5, 40.0]], np.float32)
    s = np.array([1.5, -2.0, 0.5, 1.0], np.float32)
    b = np.array([0.1, 0.0, -0.3, 0.0], np.float32)
    v = (x * s + b).astype(np.float32)
    ref = oracle.round16((v / (1.0 + np.exp(-v.astype(np.float64)))).astype(np.float32), True)
    assert np.allclose(onest.gate(x, s, b), ref, rtol=1e-3, atol=1e-6)
    qk = np.float32(1.0) / np.sqrt(np.sqrt(np.float32(32.0)))
    assert onest.attention_scale() == float(np.float32(qk * qk))
    assert abs(onest.attention_scale() - 1 / np.sqrt(32)) < 1e-7
