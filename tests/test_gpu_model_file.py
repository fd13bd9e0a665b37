"""Loading a native model file end to end on the GPU: kb_model_load_file on a
synthetic v17 TF3 file (oracle/model_file.py) evaluates bit for bit like
kb_model_load on the blob of the reference's lowering of the same layers, for
the INT8 scope and the FFN scope (binary16 attention projections)."""

import numpy as np
import pytest

import oracle.model_file as mf
from rust_katago_b200 import backend, synthetic

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("proj", [(0, 0, 0, 0), (3, 3, 0, 0)], ids=["int8", "ffn_scope"])
def test_file_model_equals_blob_model(cuda, tmp_path, proj):
    m = mf.random_native(seed=7)
    path = tmp_path / "tf3.bin.gz"
    mf.write(path, m)
    shape, blob = mf.lower(m)
    topo = synthetic.Topology(shape["trunk_channels"], shape["num_blocks"], shape["num_heads"], 32,
                              shape["ffn_channels"], proj_precision=proj, topology=1,
                              mid_channels=shape["mid_channels"], pairs_per_block=shape["pairs_per_block"],
                              norm_eps=shape["norm_eps"])
    spatial, glob = synthetic.make_positions(3, 4)
    from_file = backend.CudaBackend.load_model_file(str(path), recipe=topo)
    assert from_file.topology.mid_channels == 128 and from_file.postprocess.model_version == 17
    from_blob = backend.CudaBackend.load_model(topo, blob)
    a = backend.CudaBackend.create_compute_handle(from_file, 3).get_output(spatial, glob)
    b = backend.CudaBackend.create_compute_handle(from_blob, 3).get_output(spatial, glob)
    for f in ("policy", "value", "misc", "moremisc", "ownership"):
        assert np.array_equal(getattr(a, f), getattr(b, f)), f
    assert np.isfinite(a.policy).all()
