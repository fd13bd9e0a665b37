"""The nested (TF3) trunk on the GPU against the oracle's restatement of the
reference's lowered TF3 graph (oracle/trunk_nested.py; native_model.rs:79-165,
debug_exec_units.rs:84-380).

Every step is reproduced exactly by the oracle (binary16 tensor-core GEMMs
with the tensor cores' accumulation, INT8 projections and SwiGLU FFN, the
attention kernel's softmax, the gates), so the recorded binary16 planes (the
gated raw trunk after every outer block, and the trunk tip) are compared bit
for bit; the policy / value heads after the head linears run in fp32 on the
GPU and in float64 in the oracle, and agree to 1e-5 relative L2.
"""

import numpy as np
import pytest

import oracle.trunk_nested as onest
from rust_katago_b200 import _capi, backend, synthetic

pytestmark = pytest.mark.gpu

SMALL = synthetic.Topology(256, 2, 4, 32, 384, topology=1, mid_channels=128, pairs_per_block=2)
SMALL_FFN = synthetic.Topology(256, 2, 4, 32, 384, topology=1, mid_channels=128, pairs_per_block=2,
                               proj_precision=(3, 3, 0, 0))


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def topo_tuple(t):
    return (t.trunk_channels, t.num_blocks, t.pairs_per_block, t.num_heads, t.mid_channels, t.ffn_channels)


def run_and_compare(torch, oracle, topo, n, seed=5):
    blob = synthetic.make_blob(topo, seed)
    spatial, glob = synthetic.make_positions(n, seed + 8)
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, n)
    dsp, dgl = torch.from_numpy(spatial).cuda(), torch.from_numpy(glob).cuda()
    dout = torch.zeros(n * backend.OUT_PER_POS, device="cuda")
    trace = torch.zeros((topo.num_blocks + 2, n * 361, topo.trunk_channels), dtype=torch.int16, device="cuda")
    h.forward_trace(n, dsp, dgl, dout, trace)
    torch.cuda.synchronize()
    tr = trace.cpu().numpy().view(np.uint16)
    ref = onest.forward(blob, topo_tuple(topo), spatial, glob, attn_int8=topo.resolved_precision()[0] == "int8",
                        trace=True)
    for i, plane in enumerate(ref["trace"]):
        bits = oracle.f16_encode(plane)
        same = float(np.mean(tr[i] == bits))
        assert same == 1.0, f"plane {i}: {same:.6f} identical"
    got = backend.unpack_outputs(dout.cpu().numpy(), n)
    errs = {k: rel_l2(getattr(got, k), ref[k]) for k in ("policy", "value", "misc", "moremisc", "ownership")}
    print(topo_tuple(topo), topo.resolved_precision(), "outputs rel-L2:", {k: f"{v:.1e}" for k, v in errs.items()})
    for k, v in errs.items():
        assert v < 1e-5, k
    assert h.read_status() == (0, 0xFFFFFFFF)
    return h, spatial, glob, got


@pytest.mark.parametrize("topo", [SMALL, SMALL_FFN], ids=["int8_attention", "ffn_scope"])
def test_small_nested_bit_exact(cuda, oracle, topo):
    run_and_compare(cuda, oracle, topo, 3)


@pytest.mark.parametrize("topo", [synthetic.TF3_B11C768, synthetic.TF3_B11C768_FFN], ids=["int8_attention", "ffn_scope"])
def test_tf3_b11c768_bit_exact(cuda, oracle, topo):
    """The reference's TF3 b11c768 shape: 11 outer blocks of 3 pairs at width
    384, 12 heads x 32, SwiGLU 1152, free-running, bit for bit."""
    run_and_compare(cuda, oracle, topo, 2)


def test_nested_graph_replay_and_batch_invariance(cuda, oracle):
    topo = SMALL
    h, spatial, glob, ref = run_and_compare(cuda, oracle, topo, 4, seed=9)
    for _ in range(3):  # direct, captured, replayed
        got = h.get_output(spatial, glob)
        assert np.array_equal(got.policy, ref.policy) and np.array_equal(got.ownership, ref.ownership)
    one = h.get_output(spatial[2:3], glob[2:3])
    assert np.array_equal(one.policy[0], ref.policy[2]) and np.array_equal(one.value[0], ref.value[2])


def test_nested_rejects_unsupported(cuda):
    blob = synthetic.make_blob(SMALL, 1)
    bad = synthetic.Topology(256, 2, 4, 32, 384, topology=1, mid_channels=128, pairs_per_block=2, precision=1)
    with pytest.raises(_capi.KbError, match="KB_PREC_INT8"):
        backend.CudaBackend.load_model(bad, blob)
