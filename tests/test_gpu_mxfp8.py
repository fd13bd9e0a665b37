"""MXFP8 parity on the GPU against the CPU oracle (oracle/mxfp8.py).

Mirrors the reference's operator gates (Rust_KataGo
crates/kata_nn/tests/test_mxfp8.rs:564-1000): byte-exact quantised values and
packed scales for the conversion / scale / source-precision boundary sets,
unsafe-weight rejection, zero-weight half-edge activations, the six dyadic
shapes bit for bit and the random shapes inside the fp64 gamma bound, shared
scratch switching K (A-B-A), and the sticky status protocol.
"""

import numpy as np
import pytest

from oracle import mxfp8 as mx

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GUARD = 128
HALF_CANARY = 0x3555
FLOAT_CANARY = 0x4A123456


@pytest.fixture(scope="module")
def kb(cuda):
    from rust_katago_b200 import _capi, mxfp8

    return _capi, mxfp8


def dev_bytes(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().view(np.uint8)


def check_pack(q_dev, s_dev, expected: mx.Packed, tail_zero=True):
    q = dev_bytes(q_dev)[:expected.values.size]
    s = dev_bytes(s_dev)
    assert np.array_equal(q, expected.values.ravel()), f"FP8 bytes differ at {np.nonzero(q != expected.values.ravel())[0][:8]}"
    got = s[:expected.scales.size]
    assert np.array_equal(got, expected.scales), f"scale bytes differ at {np.nonzero(got != expected.scales)[0][:8]}"
    if tail_zero:
        assert np.all(s[expected.scales.size:] == 0), "scale scratch tail must be clear"


def check_weight(w, expected: mx.Packed):
    q, s = w.download()
    assert np.array_equal(q.ravel(), expected.values.ravel())
    assert np.array_equal(s, expected.scales)


def half_device(src_f32):
    return torch.from_numpy(mx.half_encode(src_f32).view(np.int16).copy()).cuda()


def test_conversion_boundaries_weight_bytes(kb):
    _capi, m = kb
    dec = mx.fp8_decode(np.arange(127))
    vals = []
    for code in range(126):
        mid = np.float32((dec[code] + dec[code + 1]) * 0.5)
        for v in (mx.next_down(mid), mid, mx.next_up(mid)):
            vals += [np.float32(v), np.float32(-v)]
    rows, stride = len(vals), 39
    src = np.full(rows * stride, np.nan, np.float32).reshape(rows, stride)
    src[:, :32] = 0
    src[:, 0] = 448.0
    src[:, 1] = vals
    w = m.Mxfp8Weight(src, rows, 32, stride)
    check_weight(w, mx.quantize(src, rows, 32, stride))


def test_scale_boundaries_and_subnormals(kb):
    _capi, m = kb
    maxima = [np.float32(0.0), np.float32(np.finfo(np.float32).smallest_subnormal), np.finfo(np.float32).tiny]
    for e in (-127, -126, -100, -20, 0, 20, 100, 117):
        mv = np.float32(448.0 * 2.0 ** e)
        maxima += [mx.next_down(mv), mv, mx.next_up(mv)]
    rows, stride = len(maxima), 37
    src = np.full((rows, stride), np.nan, np.float32)
    for r, mv in enumerate(maxima):
        src[r, :32] = mv
        src[r, 1] = -mv
    w = m.Mxfp8Weight(src, rows, 32, stride)
    check_weight(w, mx.quantize(src, rows, 32, stride))


def test_original_fp32_not_prerounded(kb):
    _capi, m = kb
    n, k, stride = 24, 65, 79
    src = mx.test_input(n, k, stride, 37, False, False)
    src[0] = 448.0
    src[1] = mx.next_up(np.float32(1.0625))
    src[2] = mx.next_down(np.float32(1.1875))
    src[3] = -0.0
    src[stride] = np.float32(np.finfo(np.float32).smallest_subnormal)
    expected = mx.quantize(src, n, k, stride)
    rounded = mx.half_decode(mx.half_encode(src))
    assert not np.array_equal(expected.values, mx.quantize(rounded, n, k, stride).values)
    w = m.Mxfp8Weight(src, n, k, stride)
    assert (w.n, w.k, w.kp) == (n, k, 96)
    check_weight(w, expected)


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf, np.finfo(np.float32).max])
def test_unsafe_weights_rejected(kb, bad):
    _capi, m = kb
    v = np.zeros(24 * 32, np.float32)
    v[35] = bad
    with pytest.raises(_capi.KbError) as e:
        m.Mxfp8Weight(v, 24, 32, 32)
    assert e.value.code == _capi.KB_E_NONFINITE


def test_quantizer_layout_padding_f32_and_half(kb):
    _capi, m = kb
    rows, k, stride = 129, 344, 357
    kp, _, data, scale = m.dimensions(rows, k)
    src = mx.test_input(rows, k, stride, 29, False, False)
    q = torch.full((data,), 0xAB, dtype=torch.uint8, device="cuda")
    s = torch.full((scale + 1000,), 0xCD, dtype=torch.uint8, device="cuda")
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    m.reset_status(st)
    x = torch.from_numpy(src).cuda()
    m.quantize(x, _capi.DT_F32, rows, k, stride, q, s, st)
    check_pack(q, s, mx.quantize(src, rows, k, stride))
    src_h = mx.test_input(rows, k, stride, 31, True, False)
    m.quantize(half_device(src_h), _capi.DT_F16, rows, k, stride, q, s, st)
    check_pack(q, s, mx.quantize(src_h, rows, k, stride))
    torch.cuda.synchronize()
    m.validate_status(st.cpu().numpy().view(np.uint32))


def test_zero_weights_half_edges(kb):
    _capi, m = kb
    ws = m.Mxfp8Workspace(129, 344)
    for case, k in enumerate([31, 32, 33, 65, 344, 31]):
        stride = k + 7
        zero = m.Mxfp8Weight(np.zeros(24 * k, np.float32), 24, k, k)
        src = mx.test_input(129, k, stride, 41 + case, True, False)
        if k >= 32:
            edge = [0x0001, 0x8001, 0x03FF, 0x7BFF, 0xFBFF, 0]
            src[stride:stride + k] = mx.half_decode(np.array([edge[c % 6] for c in range(k)], np.uint16))
        hx = half_device(src)
        before = hx.clone()
        out = torch.zeros(129 * 24, dtype=torch.float32, device="cuda")
        ws.begin_forward()
        ws.project(zero, hx, _capi.DT_F16, stride, out, m.OUT_FLOAT, case)
        m.validate_status(ws.status_host())
        check_pack(ws.q, ws.scales, mx.quantize(src, 129, k, stride))
        assert torch.equal(hx, before), "strided source must remain read-only"
        assert torch.all(out == 0)


def _output(mode, count, residual=None):
    if mode == 0:  # half
        t = torch.full((count + GUARD,), HALF_CANARY, dtype=torch.int16, device="cuda")
        t[:count] = 0
    else:
        t = torch.from_numpy(np.full(count + GUARD, FLOAT_CANARY, np.uint32).view(np.float32)).cuda()
        t[:count] = 0 if residual is None else torch.from_numpy(residual).cuda()
    return t


def _bits(t, mode, count):
    torch.cuda.synchronize()
    host = t.cpu().numpy()
    if mode == 0:
        assert np.all(host[count:].view(np.uint16) == HALF_CANARY), "half output tail guard"
        return host[:count].view(np.uint16)
    assert np.all(host[count:].view(np.uint32) == FLOAT_CANARY), "float output tail guard"
    return host[:count]


def gemm_case(kb, rows, n, k, mode, exact, seed):
    _capi, m = kb
    ws_, st_ = k + 13, k + 7
    weights = mx.test_input(n, k, ws_, seed, False, exact)
    act = mx.test_input(rows, k, st_, seed + 2, True, exact)
    w_ref = mx.quantize(weights, n, k, ws_)
    x_ref = mx.quantize(act, rows, k, st_)
    residual = None
    if mode == m.OUT_FLOAT_RESIDUAL:
        residual = ((np.arange(rows * n) % 17).astype(np.float32) - 8.0) * np.float32(0.25)
    exact_v, sum_abs = mx.reference(w_ref, x_ref, residual)
    if exact:
        assert np.array_equal(exact_v, exact_v.astype(np.float32).astype(np.float64))
    w = m.Mxfp8Weight(weights, n, k, ws_)
    check_weight(w, w_ref)
    ws = m.Mxfp8Workspace(rows, k)
    hx = half_device(act)
    out = _output(0 if mode == m.OUT_HALF else 1, rows * n, residual)
    ws.begin_forward()
    ws.project(w, hx, _capi.DT_F16, st_, out, mode, 7)
    m.validate_status(ws.status_host())
    check_pack(ws.q, ws.scales, x_ref)
    bits = _bits(out, 0 if mode == m.OUT_HALF else 1, rows * n)
    mx.check_output(bits, mode == m.OUT_HALF, k, exact_v, sum_abs, exact)
    check_weight(w, w_ref)
    # bit for bit against the tensor cores' block-scaled accumulation as the
    # oracle restates it (kb_oracle.c or_tc_gemm_mxf8)
    import oracle

    acc = oracle.tc_gemm_mxf8(x_ref, w_ref).ravel()
    if mode == m.OUT_HALF:
        assert np.array_equal(bits, mx.half_encode(acc)), "half output differs from the accumulation model"
    else:
        want = acc if residual is None else (residual + acc).astype(np.float32)
        assert np.array_equal(bits.view(np.uint32), want.view(np.uint32)), "fp32 output differs from the model"
    return bits


DYADIC = [(361, 136, 160, 0), (361, 384, 384, 0), (17, 384, 344, 0), (129, 24, 72, 0), (361, 136, 160, 1),
          (361, 136, 160, 2)]
RANDOM = [(361, 136, 344, 0), (17, 24, 72, 1), (129, 24, 168, 2)]


@pytest.mark.parametrize("rows,n,k,mode", DYADIC)
def test_dyadic_shapes_bitwise(kb, rows, n, k, mode):
    gemm_case(kb, rows, n, k, mode, True, 43)


@pytest.mark.parametrize("rows,n,k,mode", RANDOM)
def test_random_shapes_fp64_bound(kb, rows, n, k, mode):
    gemm_case(kb, rows, n, k, mode, False, 47)


def test_large_shape_bound(kb):
    """A trunk-sized projection (many M and N tiles, K = 768, 6 K tiles)."""
    gemm_case(kb, 2888, 3072, 768, 0, False, 71)


def test_shared_scratch_k_switches(kb):
    _capi, m = kb
    rows = 129
    ws = m.Mxfp8Workspace(rows, 344)
    sources, weights = [], []
    for index, k in enumerate([344, 344, 72, 168]):
        src = mx.test_input(24, k, k + 13, 53, False, False)
        if index == 1:
            src.reshape(24, k + 13)[:, :k] *= 8.0
        weights.append(m.Mxfp8Weight(src, 24, k, k + 13))
        sources.append(src)
    assert not np.array_equal(weights[0].download()[1], weights[1].download()[1])
    first = None
    for index in [0, 1, 2, 3, 1, 2, 0]:
        k = weights[index].k
        stride = k + 7
        act = mx.test_input(rows, k, stride, 59, True, False)
        x_ref = mx.quantize(act, rows, k, stride)
        w_ref = mx.quantize(sources[index], 24, k, k + 13)
        exact_v, sum_abs = mx.reference(w_ref, x_ref)
        out = _output(1, rows * 24)
        ws.begin_forward()
        ws.project(weights[index], half_device(act), _capi.DT_F16, stride, out, m.OUT_FLOAT, 10 + index)
        m.validate_status(ws.status_host())
        check_pack(ws.q, ws.scales, x_ref)
        bits = _bits(out, 1, rows * 24)
        mx.check_output(bits, False, k, exact_v, sum_abs, False)
        if index == 0:
            if first is None:
                first = bits.copy()
            else:
                assert np.array_equal(bits.view(np.uint32), first.view(np.uint32)), "return to large K must reproduce"
        check_weight(weights[index], w_ref)


def test_sticky_status_first_layer_and_overflow(kb):
    _capi, m = kb
    rows, n, k, stride = 17, 24, 72, 79
    w = m.Mxfp8Weight(np.ones(n * k, np.float32), n, k, k)
    ws = m.Mxfp8Workspace(rows, k)
    src = mx.test_input(rows, k, stride, 61, True, True)
    good = mx.half_encode(src)
    nan = good.copy()
    nan[stride + 3] = 0x7E00
    inf = good.copy()
    inf[2 * stride + 5] = 0xFC00
    d_good, d_nan, d_inf = (torch.from_numpy(a.view(np.int16).copy()).cuda() for a in (good, nan, inf))
    out = torch.zeros(rows * n, dtype=torch.float32, device="cuda")
    ws.begin_forward()
    for layer, x in ((3, d_good), (17, d_nan), (23, d_inf), (31, d_good)):
        ws.project(w, x, _capi.DT_F16, stride, out, m.OUT_FLOAT, layer)
    flags, first = ws.status_host()
    assert flags & 3 == 3, "later valid layer must not clear NaN/Inf bits"
    assert first == 17, "first bad layer is sticky"
    with pytest.raises(_capi.KbError):
        m.validate_status([flags, first])
    ws.begin_forward()
    ws.project(w, d_good, _capi.DT_F16, stride, out, m.OUT_FLOAT, 3)
    m.validate_status(ws.status_host())
    # Finite inputs can still overflow half storage: the whole forward fails.
    large = torch.from_numpy(np.full(rows * stride, mx.half_encode(np.float32(65504.0)), np.uint16).view(np.int16)).cuda()
    half_out = torch.zeros(rows * n, dtype=torch.int16, device="cuda")
    ws.begin_forward()
    ws.project(w, large, _capi.DT_F16, stride, half_out, m.OUT_HALF, 42)
    ws.project(w, d_good, _capi.DT_F16, stride, out, m.OUT_FLOAT, 43)
    flags, first = ws.status_host()
    assert flags & _capi.STATUS_OUTPUT_NONFINITE and first == 42
    # Host misuse is rejected before any launch.
    with pytest.raises(_capi.KbError):
        ws.project(w, d_good, _capi.DT_F16, k - 1, out, m.OUT_FLOAT, 1)


@pytest.mark.parametrize("boundary", ["bf16", "f16"])
def test_rms_mxfp8_matches_oracle(kb, oracle, boundary):
    """Fused RMSNorm -> 16-bit -> MXFP8 equals the oracle's RMSNorm (same
    summation order, rstd and rounding as the INT8 RMS quantiser) followed by
    the block-32 quantiser, byte for byte; includes a NaN row."""
    _capi, m = kb
    rows, width = 723, 768
    rng = np.random.default_rng(5)
    x = oracle.decode16(oracle.bf16_encode((rng.standard_normal((rows, width)) * 3).astype(np.float32)), False)
    x[5, 17] = np.nan
    gamma = (1 + 0.02 * rng.standard_normal(width)).astype(np.float32)
    f16 = boundary == "f16"
    _, _, normed = oracle.rms_quantize(x, gamma, 1e-6, f16)
    expected = mx.quantize(normed, rows, width, width)
    _, _, data, scale = m.dimensions(rows, width)
    q = torch.zeros(data, dtype=torch.uint8, device="cuda")
    s = torch.full((scale,), 0xEE, dtype=torch.uint8, device="cuda")
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    m.reset_status(st)
    dx = torch.from_numpy(oracle.bf16_encode(x).view(np.int16)).cuda()
    dg = torch.from_numpy(gamma).cuda()
    m.rms_quantize(dx, _capi.DT_BF16, rows, width, width, dg, 1e-6, _capi.DT_F16 if f16 else _capi.DT_BF16, q, s, st,
                   layer=9)
    check_pack(q, s, expected)
    torch.cuda.synchronize()
    flags, layer = (int(v) & 0xFFFFFFFF for v in st.cpu().tolist())
    assert flags == _capi.STATUS_NAN and layer == 9


@pytest.mark.parametrize("residual", [False, True])
def test_bf16_epilogues_bias_gelu_residual(kb, oracle, residual):
    """bf16 outputs of the trunk: bf16(gelu(acc + bias)) and bf16(r + (acc + bias)),
    acc within the fp32 accumulation bound of the exact decoded product."""
    _capi, m = kb
    rows, n, k = 777, 384, 768
    rng = np.random.default_rng(7)
    wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    xf = oracle.decode16(oracle.bf16_encode(rng.standard_normal((rows, k)).astype(np.float32)), False)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
    w = m.Mxfp8Weight(wf, n, k, k)
    _, _, data, scale = m.dimensions(rows, k)
    q = torch.zeros(data, dtype=torch.uint8, device="cuda")
    s = torch.zeros(scale, dtype=torch.uint8, device="cuda")
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    m.reset_status(st)
    m.quantize(torch.from_numpy(oracle.bf16_encode(xf).view(np.int16)).cuda(), _capi.DT_BF16, rows, k, k, q, s, st)
    r = oracle.decode16(oracle.bf16_encode(rng.standard_normal((rows, n)).astype(np.float32)), False)
    out = torch.from_numpy(oracle.bf16_encode(r).view(np.int16)).cuda() if residual else \
        torch.zeros((rows, n), dtype=torch.int16, device="cuda")
    if residual:
        m.gemm(q, s, rows, w, out, n, m.OUT_BF16_RESIDUAL, st, bias=torch.from_numpy(bias).cuda())
    else:
        m.gemm(q, s, rows, w, out, n, m.OUT_BF16, st, bias=torch.from_numpy(bias).cuda(), act=_capi.ACT_GELU)
    torch.cuda.synchronize()
    got = oracle.decode16(out.cpu().numpy().view(np.uint16), False)
    exact, _ = mx.reference(mx.quantize(wf, n, k, k), mx.quantize(xf, rows, k, k))
    v = (exact.astype(np.float32) + bias[None, :]).astype(np.float32)
    ref = oracle.decode16(oracle.bf16_encode((r + v).astype(np.float32) if residual else oracle.act(v, 1)), False)
    diff = np.abs(got.astype(np.float64) - ref)
    # one bf16 step of the larger magnitude at most, on a small fraction of outputs
    ulp = np.maximum(np.abs(ref), 1e-30) * 2.0 ** -7
    assert np.all(diff <= ulp + 1e-6)
    assert np.mean(diff > 0) < 0.02
    m.validate_status([int(v) & 0xFFFFFFFF for v in st.cpu().tolist()])
