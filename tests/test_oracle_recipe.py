"""The oracle's per-projection precision path (a precision recipe,
crates/kata_nn/src/quantization_plan.rs:36-80) against its single-precision
branches, and the host mirror's recipe resolution (cudaInt8MinFfnWidth,
crates/kata_nn/src/backends/int8.rs:73-83)."""

import numpy as np
import pytest

import oracle.trunk as otrunk
from rust_katago_b200 import _capi, synthetic

SMALL = synthetic.Topology(256, 2, 4, 64, 1024)


def topo_tuple(t):
    return (t.trunk_channels, t.num_blocks, t.num_heads, t.head_dim, t.ffn_channels)


@pytest.mark.parametrize("kind", ["int8", "mxfp8"])
def test_uniform_recipe_equals_single_precision_branch(oracle, kind):
    blob = synthetic.make_blob(SMALL, 5)
    spatial, glob = synthetic.make_positions(1, 17)
    a = otrunk.forward(blob, topo_tuple(SMALL), spatial, glob, precision=kind)
    b = otrunk.forward(blob, topo_tuple(SMALL), spatial, glob, precision=(kind,) * 4)
    for k in ("residual", "policy", "value", "ownership"):
        assert np.array_equal(a[k], b[k]), k


def test_resolution():
    P = _capi
    t = synthetic.Topology(256, 2, 4, 64, 1024)
    assert t.resolved_precision() == ("int8",) * 4
    assert synthetic.Topology(precision=1).resolved_precision() == ("mxfp8",) * 4
    ffn_only = synthetic.Topology(proj_precision=(P.PROJ_BF16, P.PROJ_BF16, 0, 0))
    assert ffn_only.resolved_precision() == ("bf16", "bf16", "int8", "int8")
    # cudaInt8MinFfnWidth: inclusive threshold on the unpadded FFN width
    assert synthetic.Topology(ffn_channels=1024, int8_min_ffn_width=1024).resolved_precision() == ("int8",) * 4
    assert synthetic.Topology(ffn_channels=1024, int8_min_ffn_width=1032).resolved_precision() == \
        ("int8", "int8", "bf16", "bf16")
    # only INT8 FFN projections are affected
    mixed = synthetic.Topology(ffn_channels=1024, int8_min_ffn_width=2048,
                               proj_precision=(0, 0, P.PROJ_MXFP8, P.PROJ_INT8))
    assert mixed.resolved_precision() == ("int8", "int8", "mxfp8", "bf16")


def test_descriptor_validation(oracle):
    """kb_model_blob_floats validates the descriptor without a GPU."""
    import ctypes

    from rust_katago_b200._capi import call, KbError

    def floats(t):
        n = ctypes.c_size_t()
        call("kb_model_blob_floats", ctypes.byref(t.desc()), ctypes.byref(n))
        return n.value

    base = floats(synthetic.Topology(256, 2, 4, 64, 1024))
    assert floats(synthetic.Topology(256, 2, 4, 64, 1024, proj_precision=(3, 2, 1, 0), int8_min_ffn_width=8)) == base
    for bad in (dict(proj_precision=(4, 0, 0, 0)), dict(proj_precision=(0, -1, 0, 0)), dict(int8_min_ffn_width=12),
                dict(int8_min_ffn_width=8200)):
        with pytest.raises(KbError):
            floats(synthetic.Topology(256, 2, 4, 64, 1024, **bad))
