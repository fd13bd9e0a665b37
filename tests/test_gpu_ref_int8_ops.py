"""This library's INT8 boundary kernels against the reference's own
int8_ops.cu, compiled unmodified for sm_100a and run on the same GPU
(oracle/ref_int8_ops.py), on the closed-form inputs of the reference's tests
(crates/kata_nn/tests/int8_kernels.rs:10-199, :329-431).

* Row quantiser (fp16 rows, both reference kernels) and the dequantisers
  (half output; fp32 residual): bit for bit.
* Fused RMSNorm -> fp16 -> INT8: the reference sums x*x one column per lane
  and takes rsqrtf; this library sums 8-column groups per lane and takes the
  correctly rounded 1/sqrt (the CPU oracle restates it exactly).  The two
  rstd differ in their last bits on some rows, which moves an fp16 boundary
  value across a rounding point now and then: every differing integer is
  listed, one step at most, and each differing scale is one fp16 step of the
  row maximum apart.
* SwiGLU requantisation: the reference computes e^-g with CUDA's expf, this
  library with its own silu_exp (a fixed IEEE sequence the oracle restates);
  the same bound and listing as for the RMS quantiser.
"""

import numpy as np
import pytest

from rust_katago_b200 import _capi, int8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(cuda):
    import oracle.ref_int8_ops as r

    if r.build() is None:
        pytest.skip("the reference's int8_ops.cu was not compiled (no reference tree and no cubin)")
    cuda.zeros(1, device="cuda")  # a current context
    return r.RefKernels()


def rms_inputs(rows, mid):
    """int8_kernels.rs:20-37: formula values with zero, 1e-18 and 1e12 rows, gamma formula."""
    i = np.arange(rows * mid)
    v = ((i * 127 + i // mid) % 997).astype(np.float32) / np.float32(191.0) - np.float32(2.5)
    kind = (i // mid) % 7
    v = np.where(kind == 0, np.float32(0), np.where(kind == 1, v * np.float32(1e-18),
                                                    np.where(kind == 2, v * np.float32(1e12), v)))
    gamma = (np.arange(mid) % 101).astype(np.float32) / np.float32(37.0) - np.float32(1.0)
    return v.astype(np.float32).reshape(rows, mid), gamma


class Ptr:
    """A raw device pointer where the bindings take a tensor."""

    def __init__(self, p):
        self.p = int(p)

    def data_ptr(self):
        return self.p


def weights(n):
    """int8_kernels.rs:130-134 / :352-356."""
    return (((np.arange(n) * 7) % 61).astype(np.float32) / np.float32(123.0) - np.float32(0.25)).astype(np.float32)


def step_diff(q_ours, q_ref, label):
    d = np.abs(q_ours.astype(np.int32) - q_ref.astype(np.int32))
    where = np.argwhere(d != 0)
    print(f"{label}: {len(where)} of {d.size} integers differ"
          + (f" (rows {sorted(set(where[:, 0].tolist()))[:12]}...)" if len(where) else ""))
    for r, c in where[:20]:
        print(f"   row {r} col {c}: ours {int(q_ours[r, c])} reference {int(q_ref[r, c])}")
    assert d.max(initial=0) <= 1
    return len(where)


def scales_close(s_ours, s_ref, label):
    same = (s_ours.view(np.uint32) == s_ref.view(np.uint32)) | (np.isnan(s_ours) & np.isnan(s_ref))
    bad = np.argwhere(~same).ravel()
    for r in bad:
        # amax is an fp16 value: one fp16 step of it, divided by 127
        amax = float(s_ref[r]) * 127.0
        step = 2.0 ** (np.floor(np.log2(amax)) - 10)
        assert abs(float(s_ours[r]) - float(s_ref[r])) * 127.0 <= step * 1.0001, (label, r, s_ours[r], s_ref[r])
    print(f"{label}: {len(bad)} of {len(s_ref)} scales differ by one fp16 step of the row maximum")
    return len(bad)


@pytest.mark.parametrize("rows,mid", [(1, 384), (361, 512), (1025, 384), (2888, 512)])
@pytest.mark.parametrize("nonfinite", [False, True])
def test_rms_quantize_vs_reference_kernel(cuda, ref, rows, mid, nonfinite):
    torch = cuda
    x, gamma = rms_inputs(rows, mid)
    if nonfinite:
        x[0, 0] = np.inf
        if rows > 1:
            x[1, 0] = np.nan
    dx, dg = torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda()
    qr = torch.zeros((rows, mid), dtype=torch.int8, device="cuda")
    sr = torch.zeros(rows, dtype=torch.float32, device="cuda")
    ref.rms_quantize(dx.data_ptr(), dg.data_ptr(), qr.data_ptr(), sr.data_ptr(), 1e-5, rows, mid)
    qo = torch.zeros((rows, mid), dtype=torch.int8, device="cuda")
    so = torch.zeros(rows, dtype=torch.float32, device="cuda")
    int8.rms_quantize(dx, _capi.DT_F32, rows, mid, mid, dg, 1e-5, _capi.DT_F16, mid, qo, so)
    torch.cuda.synchronize()
    q_ours, q_ref = qo.cpu().numpy(), qr.cpu().numpy()
    s_ours, s_ref = so.cpu().numpy(), sr.cpu().numpy()
    n_q = step_diff(q_ours, q_ref, f"RMS {rows}x{mid}")
    n_s = scales_close(s_ours, s_ref, f"RMS {rows}x{mid}")
    assert n_q <= 0.002 * q_ref.size + 4 and n_s <= 0.01 * rows + 2
    if nonfinite:
        bad = [0] + ([1] if rows > 1 else [])
        assert np.isnan(s_ours[bad]).all() and np.isnan(s_ref[bad]).all()
        assert not q_ours[bad].any() and not q_ref[bad].any()


@pytest.mark.parametrize("rows,width", [(1, 512), (1025, 128), (1025, 472), (1025, 520), (3, 1160), (3, 1152),
                                        (3, 1536), (361, 384)])
@pytest.mark.parametrize("warp", [False, True], ids=["cta256", "warp4"])
def test_quantize_rows_bitwise_vs_reference_kernel(cuda, oracle, ref, rows, width, warp):
    torch = cuda
    i = np.arange(rows * width)
    v = np.where(i < width, 0.0, (i % 97) / 43.0 - 1.0).astype(np.float32).reshape(rows, width)
    if rows > 2:
        v[2, 5] = np.inf
    x16 = oracle.f16_encode(v)
    kp = (width + 15) // 16 * 16
    dx = torch.from_numpy(x16.view(np.int16)).cuda()
    qr = torch.full((rows, kp), 99, dtype=torch.int8, device="cuda")
    sr = torch.zeros(rows, dtype=torch.float32, device="cuda")
    ref.quantize_rows(dx.data_ptr(), qr.data_ptr(), sr.data_ptr(), rows, width, width, kp, warp)
    qo = torch.full((rows, kp), 99, dtype=torch.int8, device="cuda")
    so = torch.zeros(rows, dtype=torch.float32, device="cuda")
    int8.quantize_rows(dx, _capi.DT_F16, rows, width, width, kp, qo, so)
    torch.cuda.synchronize()
    assert np.array_equal(qo.cpu().numpy(), qr.cpu().numpy())
    a, b = so.cpu().numpy(), sr.cpu().numpy()
    assert np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(a[~np.isnan(a)].view(np.uint32),
                                                                         b[~np.isnan(b)].view(np.uint32))


@pytest.mark.parametrize("rows,mid,hidden", [(1025, 512, 128), (1025, 512, 472), (3, 512, 1160), (3, 384, 1152),
                                             (361, 384, 512)])
def test_swiglu_requant_vs_reference_kernel(cuda, oracle, ref, rows, mid, hidden):
    """Dual GEMM int32 dots -> the reference's SwiGLU requantiser, against this
    library's SwiGLU epilogue (kb_int8_linear KB_EPI_SWIGLU16) -> fp16 hidden ->
    kb_int8_quantize_rows, with the same activation scales."""
    torch = cuda
    i = np.arange(rows * mid)
    xv = np.where(i < mid, 0.0, (i % 97) / 43.0 - 1.0).astype(np.float32).reshape(rows, mid)
    x16 = oracle.f16_encode(xv)
    dual_w = weights(2 * hidden * mid).reshape(2 * hidden, mid)
    plain = int8.Int8Weight(dual_w)
    dual = int8.Int8Weight(dual_w, _capi.LAYOUT_SWIGLU_DUAL)
    kpm, kph = (mid + 15) // 16 * 16, (hidden + 15) // 16 * 16
    dx = torch.from_numpy(x16.view(np.int16)).cuda()
    qa = torch.zeros((rows, kpm), dtype=torch.int8, device="cuda")
    sa = torch.zeros(rows, dtype=torch.float32, device="cuda")
    int8.quantize_rows(dx, _capi.DT_F16, rows, mid, mid, kpm, qa, sa)
    # reference: int32 dots [rows, 2H] ([gate | up]) -> its requantiser (overwrites the scales)
    dots = torch.zeros((rows, 2 * hidden), dtype=torch.int32, device="cuda")
    int8.gemm_i32(qa, Ptr(plain.q_ptr), dots, rows, 2 * hidden, kpm)
    sr = sa.clone()
    qr = torch.zeros((rows, kph), dtype=torch.int8, device="cuda")
    warp = hidden <= 512 and rows >= 64
    ref.swiglu_quantize(dots.data_ptr(), sr.data_ptr(), plain.scales_ptr, qr.data_ptr(), rows, hidden, kph, warp)
    # this library: SwiGLU epilogue -> fp16 hidden -> row quantiser
    hid = torch.zeros((rows, hidden), dtype=torch.int16, device="cuda")
    int8.linear(qa, sa, Ptr(dual.q_ptr), Ptr(dual.scales_ptr), None, rows, dual.n_stored, kpm, _capi.EPI_SWIGLU16,
                hid, hidden, out_dtype=_capi.DT_F16, n_out=hidden)
    qo = torch.zeros((rows, kph), dtype=torch.int8, device="cuda")
    so = torch.zeros(rows, dtype=torch.float32, device="cuda")
    int8.quantize_rows(hid, _capi.DT_F16, rows, hidden, hidden, kph, qo, so)
    torch.cuda.synchronize()
    n_q = step_diff(qo.cpu().numpy(), qr.cpu().numpy(), f"SwiGLU {rows}x{mid}x{hidden}")
    n_s = scales_close(so.cpu().numpy(), sr.cpu().numpy(), f"SwiGLU {rows}x{mid}x{hidden}")
    assert n_q <= 0.002 * rows * kph + 4 and n_s <= 0.01 * rows + 2


@pytest.mark.parametrize("residual", [False, True], ids=["half", "residual"])
def test_dequantisers_bitwise_vs_reference_kernels(cuda, oracle, ref, residual):
    torch = cuda
    rows, n, k = 361, 384, 512
    rng = np.random.default_rng(3)
    a = rng.integers(-127, 128, (rows, k), dtype=np.int8)
    w = rng.integers(-127, 128, (n, k), dtype=np.int8)
    sa = (rng.random(rows) * 0.01 + 1e-3).astype(np.float32)
    sw = (rng.random(n) * 0.01 + 1e-3).astype(np.float32)
    da, dw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    dsa, dsw = torch.from_numpy(sa).cuda(), torch.from_numpy(sw).cuda()
    dots = torch.zeros((rows, n), dtype=torch.int32, device="cuda")
    int8.gemm_i32(da, dw, dots, rows, n, k)
    if residual:
        base = ((np.arange(rows * n) % 17) * 0.25 - 2.0).astype(np.float32).reshape(rows, n)
        outr = torch.from_numpy(base.copy()).cuda()
        outo = torch.from_numpy(base.copy()).cuda()
        epi = _capi.EPI_RES_F32
    else:
        outr = torch.zeros((rows, n), dtype=torch.int16, device="cuda")
        outo = torch.zeros((rows, n), dtype=torch.int16, device="cuda")
        epi = _capi.EPI_F16
    ref.dequantize(dots.data_ptr(), dsa.data_ptr(), dsw.data_ptr(), outr.data_ptr(), rows, n, residual)
    int8.linear(da, dsa, dw, dsw, None, rows, n, k, epi, outo, n)
    torch.cuda.synchronize()
    assert np.array_equal(outo.cpu().numpy().view(np.uint32 if residual else np.uint16),
                          outr.cpu().numpy().view(np.uint32 if residual else np.uint16))
