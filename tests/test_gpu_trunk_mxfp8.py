"""MXFP8 trunk (KB_PREC_MXFP8) on the GPU against the CPU oracle's MXFP8 forward.

Every trunk projection runs as block-32 E4M3 x E4M3 with UE8M0 scales and fp32
accumulation; the oracle restates the tensor cores' block-scaled accumulation,
the attention kernel and the bf16 GEMMs exactly, so the trunk is compared bit
for bit.
"""

import numpy as np
import pytest

import oracle.trunk as otrunk
from rust_katago_b200 import backend, synthetic

pytestmark = pytest.mark.gpu

SMALL_MX = synthetic.Topology(256, 2, 4, 64, 1024, precision=1)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def topo_tuple(t):
    return (t.trunk_channels, t.num_blocks, t.num_heads, t.head_dim, t.ffn_channels)


def run(topo, blob, spatial, glob):
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, spatial.shape[0])
    return h.get_output(spatial, glob), h, model


def errors(got, ref):
    return {k: rel_l2(getattr(got, k), ref[k]) for k in ("policy", "value", "misc", "moremisc", "ownership")}


@pytest.mark.parametrize("topo,n", [(SMALL_MX, 3), (synthetic.B11C768_MXFP8, 2)], ids=["c256h64", "b11c768"])
def test_mxfp8_trunk_matches_oracle(cuda, oracle, topo, n):
    """Free-running MXFP8 forward (BASELINE config 4's model) bit for bit: the
    oracle restates the block-scaled accumulation of the tensor cores
    (or_tc_gemm_mxf8), so the final residual stream is identical and the heads
    (the trunk tip's fast SiLU, fp32 on the GPU, float64 in the oracle) agree
    to 1e-4."""
    torch = cuda
    blob = synthetic.make_blob(topo, 5)
    spatial, glob = synthetic.make_positions(n, 17)
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, n)
    dsp, dgl = torch.from_numpy(spatial).cuda(), torch.from_numpy(glob).cuda()
    dout = torch.zeros(n * backend.OUT_PER_POS, device="cuda")
    trace = torch.zeros((topo.num_blocks + 2, n * 361, topo.trunk_channels), dtype=torch.bfloat16, device="cuda")
    h.forward_trace(n, dsp, dgl, dout, trace)
    torch.cuda.synchronize()
    tr = trace.float().cpu().numpy()
    ref = otrunk.forward(blob, topo_tuple(topo), spatial, glob, precision="mxfp8")
    same = float(np.mean(tr[-1] == ref["residual"]))
    got = backend.unpack_outputs(dout.cpu().numpy(), n)
    e = errors(got, ref)
    print("MXFP8 trunk: identical residual", same, "outputs rel-L2", {k: f"{v:.1e}" for k, v in e.items()})
    assert same == 1.0
    for k, v in e.items():
        assert v < 1e-4, k
    assert h.read_status() == (0, 0xFFFFFFFF)


def test_mxfp8_batch_invariance_and_graph(cuda):
    topo = synthetic.B11C768_MXFP8
    blob = synthetic.make_blob(topo, 1234)
    spatial, glob = synthetic.make_positions(8, 21)
    got, h, _ = run(topo, blob, spatial, glob)
    again = h.get_output(spatial, glob)
    third = h.get_output(spatial, glob)
    for o in (again, third):
        assert np.array_equal(o.policy, got.policy) and np.array_equal(o.ownership, got.ownership)
    for i in (0, 5):
        one = h.get_output(spatial[i:i + 1], glob[i:i + 1])
        assert np.array_equal(one.policy[0], got.policy[i])
        assert np.array_equal(one.value[0], got.value[i])
    assert h.read_status() == (0, 0xFFFFFFFF)


def test_mxfp8_vs_int8_same_weights(cuda):
    """Config 4 against config 3 on the same seeded weights and positions: the
    two quantisations differ (E4M3 per 32 values vs INT8 per token), so the
    outputs differ at the few-percent level; pooled value outputs stay close."""
    blob = synthetic.make_blob(synthetic.B11C768, 1234)
    spatial, glob = synthetic.make_positions(4, 3)
    mx, _, _ = run(synthetic.B11C768_MXFP8, blob, spatial, glob)
    i8, _, _ = run(synthetic.B11C768, blob, spatial, glob)
    e = errors(mx, {k: getattr(i8, k) for k in ("policy", "value", "misc", "moremisc", "ownership")})
    print("MXFP8 vs INT8 relative L2:", {k: round(v, 5) for k, v in e.items()})
    assert e["policy"] < 0.15 and e["value"] < 0.05
