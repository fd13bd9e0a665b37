"""Per-projection precision recipes (crates/kata_nn/src/quantization_plan.rs:36-80:
each of qkv / out / ffn_up / ffn_down in INT8, MXFP8 or unquantised; the
reference's unquantised projections are FP16, here bf16) and cudaInt8MinFfnWidth
(crates/kata_nn/src/backends/int8.rs:73-83) on the GPU against the oracle's
per-projection forward.

Every projection kind (INT8, MXFP8 block-scaled, bf16) and the attention
kernel are restated exactly by the oracle (the tensor cores' accumulation
included), so the residual stream is compared bit for bit, free-running and
under teacher forcing; the heads agree to 1e-4.
"""

import numpy as np
import pytest

import oracle.trunk as otrunk
from rust_katago_b200 import _capi, backend, synthetic

pytestmark = pytest.mark.gpu

P = _capi
RECIPES = {
    "ffn_scope": dict(proj_precision=(P.PROJ_BF16, P.PROJ_BF16, 0, 0)),  # Int8Scope::Ffn
    "all_bf16": dict(proj_precision=(P.PROJ_BF16,) * 4),
    "mx_i8_bf_mx": dict(proj_precision=(P.PROJ_MXFP8, P.PROJ_INT8, P.PROJ_BF16, P.PROJ_MXFP8)),
    "i8_mx_mx_i8": dict(proj_precision=(P.PROJ_INT8, P.PROJ_MXFP8, P.PROJ_MXFP8, P.PROJ_INT8)),
    "min_ffn_width": dict(int8_min_ffn_width=2048),  # F = 1024 < 2048: FFN unquantised
    "mxfp8_base_bf16_out": dict(precision=1, proj_precision=(0, P.PROJ_BF16, 0, 0)),
}


def topo_of(name):
    return synthetic.Topology(256, 2, 4, 64, 1024, **RECIPES[name])


def topo_tuple(t):
    return (t.trunk_channels, t.num_blocks, t.num_heads, t.head_dim, t.ffn_channels)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", list(RECIPES))
def test_recipe_trunk_matches_oracle(cuda, oracle, name):
    topo = topo_of(name)
    blob = synthetic.make_blob(topo, 5)
    spatial, glob = synthetic.make_positions(2, 17)
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, 2)
    got = h.get_output(spatial, glob)
    ref = otrunk.forward(blob, topo_tuple(topo), spatial, glob, precision=topo.resolved_precision())
    e = {k: rel_l2(getattr(got, k), ref[k]) for k in ("policy", "value", "misc", "moremisc", "ownership")}
    print(name, topo.resolved_precision(), {k: f"{v:.1e}" for k, v in e.items()})
    for k, v in e.items():
        assert v < 1e-4, k
    assert h.read_status() == (0, 0xFFFFFFFF)


@pytest.mark.parametrize("name", ["ffn_scope", "mx_i8_bf_mx"])
def test_recipe_teacher_forced_and_graph(cuda, oracle, name):
    torch = cuda
    topo = topo_of(name)
    n = 2
    blob = synthetic.make_blob(topo, 5)
    spatial, glob = synthetic.make_positions(n, 13)
    model = backend.CudaBackend.load_model(topo, blob)
    h = backend.CudaBackend.create_compute_handle(model, n)
    dsp, dgl = torch.from_numpy(spatial).cuda(), torch.from_numpy(glob).cuda()
    dout = torch.zeros(n * backend.OUT_PER_POS, device="cuda")
    trace = torch.zeros((topo.num_blocks + 2, n * 361, topo.trunk_channels), dtype=torch.bfloat16, device="cuda")
    h.forward_trace(n, dsp, dgl, dout, trace)
    torch.cuda.synchronize()
    tr = trace.float().cpu().numpy()
    ref = otrunk.forward(blob, topo_tuple(topo), spatial, glob, precision=topo.resolved_precision(),
                         teacher=(tr[0], [tr[1 + i] for i in range(topo.num_blocks)]))
    res_err = rel_l2(tr[-1], ref["residual"])
    print(name, f"teacher-forced residual rel-L2 {res_err:.2e}, identical {np.mean(tr[-1] == ref['residual']):.4f}")
    assert np.array_equal(tr[-1], ref["residual"])
    # the graph path (kb_submit) gives the trace forward's outputs bit for bit
    got = h.get_output(spatial, glob)
    flat = dout.cpu().numpy()
    ref_out = backend.unpack_outputs(flat, n)
    assert np.array_equal(got.policy, ref_out.policy) and np.array_equal(got.ownership, ref_out.ownership)


def test_recipes_share_weights_and_differ_only_by_precision(cuda):
    """All-INT8, FFN-scope and all-bf16 builds of the same weights: each loads
    and runs, their policies differ (the precisions differ) and stay close to
    one another (the model is the same)."""
    spatial, glob = synthetic.make_positions(1, 3)
    outs = []
    for kw in ({}, RECIPES["ffn_scope"], RECIPES["all_bf16"]):
        topo = synthetic.Topology(256, 2, 4, 64, 1024, **kw)
        blob = synthetic.make_blob(topo, 5)
        model = backend.CudaBackend.load_model(topo, blob)
        h = backend.CudaBackend.create_compute_handle(model, 1)
        outs.append(h.get_output(spatial, glob).policy)
    assert not np.array_equal(outs[0], outs[1]) and not np.array_equal(outs[1], outs[2])
    assert rel_l2(outs[1], outs[2]) < 5e-2 and rel_l2(outs[0], outs[2]) < 5e-2
