"""GPU test of kb_int8_ffn_gelu_rms_noalloc, the FFN entry point that allocates
nothing (for callers that cannot call cudaMalloc where they evaluate, such as a
search thread mid-move or a host with a fixed device-memory budget).

Its output must equal the workspace-based kb_int8_ffn_gelu_rms bit for bit, on
two calls in a row (the second call finds the first call's data in the shared
static scratch); further calls must leave the device's free memory unchanged;
oversize calls and weights of another device must be rejected.
Named to be collected last; it passes alone in a fresh process too.
"""

import numpy as np
import pytest

from rust_katago_b200 import _capi, int8

pytestmark = pytest.mark.gpu


def make_block(rows, c=768, f=3072, seed=11):
    rng = np.random.default_rng(seed)
    import torch

    x = torch.from_numpy(rng.standard_normal((rows, c)).astype(np.float32)).to(torch.bfloat16)
    gamma = (1 + 0.02 * rng.standard_normal(c)).astype(np.float32)
    up_w = (0.02 * rng.standard_normal((f, c))).astype(np.float32)
    down_w = (0.02 * rng.standard_normal((c, f))).astype(np.float32)
    up_b = (0.02 * rng.standard_normal(f)).astype(np.float32)
    down_b = (0.02 * rng.standard_normal(c)).astype(np.float32)
    return x, gamma, up_w, down_w, up_b, down_b


@pytest.mark.parametrize("rows", [361, 722])
def test_noalloc_matches_workspace_twice(cuda, rows):
    torch = cuda
    x, gamma, up_w, down_w, up_b, down_b = make_block(rows)
    up, down = int8.Int8Weight(up_w), int8.Int8Weight(down_w)
    g, ub, db = (torch.from_numpy(a).cuda() for a in (gamma, up_b, down_b))
    ws = int8.Int8Workspace(rows, 3072, 3072)
    ref = x.cuda()
    ws.ffn_gelu_rms(g, 1e-6, up, ub, down, db, ref, rows)
    ws.ffn_gelu_rms(g, 1e-6, up, ub, down, db, ref, rows)  # two blocks in a row
    got = x.cuda()
    int8.noalloc_prepare()
    int8.ffn_gelu_rms_noalloc(g, 1e-6, up, ub, down, db, got, rows)
    torch.cuda.synchronize()
    int8.ffn_gelu_rms_noalloc(g, 1e-6, up, ub, down, db, got, rows)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_noalloc_allocates_nothing(cuda):
    """After a first call (which may load the module's kernels), more calls do
    not change the device's free memory: the entry point's scratch is the
    static array reserved at library load."""
    torch = cuda
    rows = 361
    x, gamma, up_w, down_w, up_b, down_b = make_block(rows, seed=3)
    up, down = int8.Int8Weight(up_w), int8.Int8Weight(down_w)
    g, ub, db = (torch.from_numpy(a).cuda() for a in (gamma, up_b, down_b))
    r = x.cuda()
    int8.ffn_gelu_rms_noalloc(g, 1e-6, up, ub, down, db, r, rows)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        int8.ffn_gelu_rms_noalloc(g, 1e-6, up, ub, down, db, r, rows)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_noalloc_rejects_oversize(cuda):
    torch = cuda
    rows = 4 * 361
    x, gamma, up_w, down_w, up_b, down_b = make_block(8)
    up, down = int8.Int8Weight(up_w), int8.Int8Weight(down_w)
    resid = torch.zeros((rows, 768), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_capi.KbError, match="fixed scratch is 8388608 bytes"):
        int8.ffn_gelu_rms_noalloc(torch.from_numpy(gamma).cuda(), 1e-6, up, None, down, None, resid, rows)


def test_noalloc_rejects_weights_of_another_device(cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    x, gamma, up_w, down_w, up_b, down_b = make_block(8)
    up, down = int8.Int8Weight(up_w), int8.Int8Weight(down_w)  # on device 0
    with torch.cuda.device(1):
        resid = torch.zeros((361, 768), dtype=torch.bfloat16, device="cuda:1")
        g = torch.from_numpy(gamma).to("cuda:1")
        with pytest.raises(_capi.KbError, match="another device"):
            int8.ffn_gelu_rms_noalloc(g, 1e-6, up, None, down, None, resid, 361)
