"""The native model-file loader (kb_model_file_parse; host code, no GPU) on
synthetic v17 TF3 files (oracle/model_file.py writes them as the reference's
parser reads them): the descriptor and the weight blob equal, bit for bit,
an independent restatement of the reference's lowering, from binary, gzip and
text files alike; files the reference's native CUDA path rejects are
rejected with the reason."""

import ctypes

import numpy as np
import pytest

import oracle.model_file as mf
from rust_katago_b200 import _capi


def parse(path):
    desc = _capi.ModelDesc()
    count = ctypes.c_size_t()
    pp = _capi.PostProcessParams()
    _capi.call("kb_model_file_parse", str(path).encode(), ctypes.byref(desc), None, 0, ctypes.byref(count),
               ctypes.byref(pp))
    blob = np.zeros(count.value, np.float32)
    _capi.call("kb_model_file_parse", str(path).encode(), ctypes.byref(desc), blob.ctypes.data, blob.size,
               ctypes.byref(count), None)
    return desc, blob, pp


@pytest.mark.parametrize("suffix", [".bin.gz", ".bin", ".txt", ".txt.gz"])
def test_round_trip_matches_reference_lowering(tmp_path, suffix):
    m = mf.random_native(seed=3)
    path = tmp_path / ("model" + suffix)
    mf.write(path, m)
    desc, blob, pp = parse(path)
    shape, want = mf.lower(m)
    for k, v in shape.items():
        assert getattr(desc, k) == (np.float32(v) if k == "norm_eps" else v), k
    assert desc.topology == _capi.TOPO_NESTED and desc.precision == _capi.PREC_INT8
    assert blob.size == want.size
    assert np.array_equal(blob.view(np.uint32), want.view(np.uint32))
    assert pp.model_version == 17 and pp.lead_multiplier == 20.0 and pp.shortterm_score_error_multiplier == 30.0


def test_tf3_b11c768_shape(tmp_path):
    """The shipped TF3 b11c768 shape: 11 outer blocks of 3 pairs, mid 384, SwiGLU 1152."""
    m = mf.random_native(c=768, nb=11, pairs=3, mid=384, hidden=1152, seed=1, policy_channels=4)
    path = tmp_path / "b11c768.bin.gz"
    mf.write(path, m)
    desc, blob, _ = parse(path)
    assert (desc.trunk_channels, desc.num_blocks, desc.pairs_per_block, desc.mid_channels, desc.num_heads,
            desc.ffn_channels) == (768, 11, 3, 384, 12, 1152)
    assert np.array_equal(blob, mf.lower(m)[1])


@pytest.mark.parametrize("case,msg", [
    ("version", "version 17"),
    ("activation", "SiLU"),
    ("head_scale", "unit BN scales"),
    ("truncated", "truncated|end of file"),
    ("trailing", "trailing"),
    ("extension", "extension"),
    ("missing", "cannot open"),
])
def test_rejections(tmp_path, case, msg):
    m = mf.random_native(seed=5)
    path = tmp_path / "model.bin"
    if case == "version":
        path.write_bytes(mf.serialise(m, version=16))
    elif case == "activation":
        path.write_bytes(mf.serialise(m, activation="ACTIVATION_MISH"))
    elif case == "head_scale":
        m["p1_bn"]["scale"] = m["p1_bn"]["scale"] * np.float32(2.0)
        mf.write(path, m)
    elif case == "truncated":
        path.write_bytes(mf.serialise(m)[:-4000])
    elif case == "trailing":
        path.write_bytes(mf.serialise(m) + b"extra")
    elif case == "extension":
        path = tmp_path / "model.onnx"
        path.write_bytes(mf.serialise(m))
    else:
        path = tmp_path / "absent.bin"
    with pytest.raises(_capi.KbError, match=msg):
        parse(path)
