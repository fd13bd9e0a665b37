"""GPU parity tests of the INT8 path through the C ABI against the CPU oracle.

Bar: bit-exact.  Integer accumulators, quantised activations, scales and every
dequantised / activated / residual output are compared bitwise, because each
product kernel performs the same IEEE-rounded operation sequence as the oracle.
"""

import numpy as np
import pytest

from rust_katago_b200 import _capi, int8

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "int8_dot_cases.npz"


def dev(torch, a: np.ndarray):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t, dtype=None):
    a = t.cpu().numpy()
    return a.view(dtype) if dtype is not None else a


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def same_f32(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return bool(np.all((bits(a) == bits(b)) | (np.isnan(a) & np.isnan(b))))


# ------------------------------------------------------------------ integer GEMM
GEMM_SHAPES = [(1, 16, 16), (3, 48, 32), (65, 72, 48), (1025, 48, 32), (3, 944, 512), (2, 512, 480),
               (3, 1536, 512), (4, 2304, 384), (129, 136, 160), (361, 1152, 384), (300, 384, 1152),
               (2888, 3072, 768), (1000, 768, 3072)]


@pytest.mark.parametrize("m,n,kp", GEMM_SHAPES)
def test_gemm_i32_bit_exact(cuda, oracle, m, n, kp):
    torch = cuda
    rng = np.random.default_rng(m * 131 + n * 7 + kp)
    a = rng.integers(-127, 128, (m, kp), dtype=np.int8)
    w = rng.integers(-127, 128, (n, kp), dtype=np.int8)
    a[0] = 127  # extreme row: |dot| up to 127*127*kp
    w[0] = -127
    dots = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    int8.gemm_i32(dev(torch, a), dev(torch, w), dots, m, n, kp)
    torch.cuda.synchronize()
    assert (host(dots) == oracle.igemm(a, w)).all()


@pytest.mark.parametrize("shape", [tuple(s) for s in np.load(GOLDEN)["shapes"]])
def test_projection_cases_of_reference(cuda, oracle, shape):
    """int8_kernels.rs:224-327 cases: quantised rows, half and fp32-residual outputs bitwise."""
    torch = cuda
    rows, n, k = shape
    g = np.load(GOLDEN)
    key = f"{rows}_{n}_{k}_"
    stride = (k + 15) // 16 * 16
    weight = int8.Int8Weight(g[key + "w"])
    assert weight.kp == stride
    ws = int8.Int8Workspace(rows, stride, n)
    x = dev(torch, g[key + "x16"])
    out = torch.zeros((rows, n), dtype=torch.int16, device="cuda")
    res = dev(torch, g[key + "initial"])
    ws.project_half(x, stride, weight, out, rows)
    ws.project_residual(x, stride, weight, res, rows)
    torch.cuda.synchronize()
    assert (host(out, np.uint16) == g[key + "half"]).all()
    assert same_f32(host(res), g[key + "residual"])
    # the workspace holds the last quantised rows: zero padding and scales
    q = torch.empty((rows, stride), dtype=torch.int8, device="cuda")
    int8.quantize_rows(x, _capi.DT_F16, rows, k, stride, stride, q, torch.empty(rows, device="cuda"))
    torch.cuda.synchronize()
    qh = host(q)
    assert (qh[:, :k] == g[key + "q"]).all() and (qh[:, k:] == 0).all()


def test_project_errors(cuda):
    torch = cuda
    w = int8.Int8Weight(np.ones((16, 32), np.float32))
    ws = int8.Int8Workspace(8, 32, 16)
    x = torch.zeros((8, 32), dtype=torch.int16, device="cuda")
    out = torch.zeros((8, 16), dtype=torch.int16, device="cuda")
    other = torch.cuda.Stream()
    with pytest.raises(_capi.KbError, match="another CUDA stream"):
        ws.project_half(x, 32, w, out, 8, stream=other)
    with pytest.raises(_capi.KbError, match="rows"):
        ws.project_half(x, 32, w, out, 0)
    with pytest.raises(_capi.KbError, match="rows"):
        ws.project_half(x, 32, w, out, 9)
    with pytest.raises(_capi.KbError, match="stride"):
        ws.project_half(x, 16, w, out, 8)


# ------------------------------------------------------------------ quantisers
def rms_input(rows, mid):
    # crates/kata_nn/tests/int8_kernels.rs:21-33 (+ non-finite rows :66-75)
    i = np.arange(rows * mid)
    v = ((i * 127 + i // mid) % 997).astype(np.float32) / np.float32(191.0) - np.float32(2.5)
    kind = (i // mid) % 7
    v = np.where(kind == 0, 0.0, np.where(kind == 1, v * np.float32(1e-18), np.where(kind == 2, v * np.float32(1e12), v)))
    return v.astype(np.float32).reshape(rows, mid)


@pytest.mark.parametrize("rows,mid", [(1, 384), (361, 512), (1025, 384), (2888, 512), (23104, 768), (17, 128),
                                      (33, 256)])
@pytest.mark.parametrize("boundary", [_capi.DT_F16, _capi.DT_BF16])
@pytest.mark.parametrize("nonfinite", [False, True])
def test_rms_quantize_bit_exact(cuda, oracle, rows, mid, boundary, nonfinite):
    """fp32 rows: widths of 128..512 columns take the two-rows-per-warp kernel,
    768 the warp-per-row one; zero, tiny, huge and non-finite rows."""
    torch = cuda
    x = rms_input(rows, mid)
    if nonfinite:
        x[0, 0] = np.inf
        if rows > 1:
            x[1, 0] = np.nan
    gamma = ((np.arange(mid) % 101).astype(np.float32) / np.float32(37.0) - 1).astype(np.float32)
    kp = (mid + 15) // 16 * 16
    q = torch.full((rows, kp), 77, dtype=torch.int8, device="cuda")
    s = torch.zeros(rows, device="cuda")
    int8.rms_quantize(dev(torch, x), _capi.DT_F32, rows, mid, mid, dev(torch, gamma), 1e-5, boundary, kp, q, s)
    torch.cuda.synchronize()
    oq, os_, _ = oracle.rms_quantize(x, gamma, 1e-5, boundary == _capi.DT_F16, kp=kp)
    assert (host(q) == oq).all()
    assert same_f32(host(s), os_)


@pytest.mark.parametrize("mid,stride", [(256, 256), (512, 512), (768, 768), (1024, 1024), (768, 776), (384, 384)])
@pytest.mark.parametrize("dtype", [_capi.DT_BF16, _capi.DT_F16])
@pytest.mark.parametrize("boundary", [_capi.DT_F16, _capi.DT_BF16])
@pytest.mark.parametrize("rows", [3001, 361])
def test_rms_quantize_16bit_input_bit_exact(cuda, oracle, mid, stride, dtype, boundary, rows):
    """16-bit residual rows (the trunk's case): full rows of 256*G columns take
    the kernels without bounds checks (two rows per warp from 2048 rows, one
    below), other widths and strides the generic one; all against the oracle,
    with zero, tiny, huge and non-finite rows."""
    torch = cuda
    x = np.zeros((rows, stride), np.float32)
    x[:, :mid] = rms_input(rows, mid)
    x[0, 0], x[1, 3], x[2, mid - 1] = np.inf, np.nan, -np.inf
    f16 = dtype == _capi.DT_F16
    xb = oracle.f16_encode(x) if f16 else oracle.bf16_encode(x)
    xv = oracle.decode16(xb, f16)
    gamma = ((np.arange(mid) % 101).astype(np.float32) / np.float32(37.0) - 1).astype(np.float32)
    kp = (mid + 15) // 16 * 16
    q = torch.full((rows, kp), 77, dtype=torch.int8, device="cuda")
    s = torch.zeros(rows, device="cuda")
    int8.rms_quantize(dev(torch, xb), dtype, rows, mid, stride, dev(torch, gamma), 1e-5, boundary, kp, q, s)
    torch.cuda.synchronize()
    oq, os_, _ = oracle.rms_quantize(np.ascontiguousarray(xv[:, :mid]), gamma, 1e-5, boundary == _capi.DT_F16, kp=kp)
    assert (host(q) == oq).all()
    assert same_f32(host(s), os_)


@pytest.mark.parametrize("dtype", [_capi.DT_F16, _capi.DT_BF16, _capi.DT_F32])
@pytest.mark.parametrize("rows,width,stride", [(1, 8, 8), (3, 24, 32), (1025, 472, 480), (2000, 3072, 3072), (7, 1160, 1163)])
def test_quantize_rows_bit_exact(cuda, oracle, dtype, rows, width, stride):
    torch = cuda
    rng = np.random.default_rng(rows + width)
    x = (rng.standard_normal((rows, stride)) * rng.uniform(0.01, 100, (rows, 1))).astype(np.float32)
    x[0] = 0.0
    if dtype == _capi.DT_F16:
        xb = oracle.f16_encode(x)
        xv = oracle.decode16(xb, True)
        xd = dev(torch, xb)
    elif dtype == _capi.DT_BF16:
        xb = oracle.bf16_encode(x)
        xv = oracle.decode16(xb, False)
        xd = dev(torch, xb)
    else:
        xv = x
        xd = dev(torch, x)
    kp = (width + 15) // 16 * 16
    q = torch.full((rows, kp), 55, dtype=torch.int8, device="cuda")
    s = torch.zeros(rows, device="cuda")
    int8.quantize_rows(xd, dtype, rows, width, stride, kp, q, s)
    torch.cuda.synchronize()
    oq, os_ = oracle.quantize_rows(np.ascontiguousarray(xv[:, :width]), kp=kp)
    assert (host(q) == oq).all()
    assert same_f32(host(s), os_)


@pytest.mark.parametrize("rows,width", [(1, 8), (361, 3072), (1000, 472), (92416, 3072), (4099, 384),
                                        (2048, 256), (2049, 128), (2047, 384), (2049, 1152)])
@pytest.mark.parametrize("f16", [False, True])
def test_gemm_row_amax_and_streaming_quantiser(cuda, oracle, rows, width, f16):
    """GEMM epilogue row_amax + streaming quantiser == full-row quantiser
    (bitwise); rows of 128..384 or 1152 columns from 2048 rows take the
    two-rows-per-warp kernel."""
    torch = cuda
    odt = _capi.DT_F16 if f16 else _capi.DT_BF16
    rng = np.random.default_rng(rows + width)
    kp = 768
    a = torch.from_numpy(rng.integers(-127, 128, (rows, kp), dtype=np.int8)).cuda()
    w = torch.from_numpy(rng.integers(-127, 128, (width, kp), dtype=np.int8)).cuda()
    sa = torch.from_numpy(rng.uniform(1e-4, 1e-2, rows).astype(np.float32)).cuda()
    sw = torch.from_numpy(rng.uniform(1e-4, 1e-2, width).astype(np.float32)).cuda()
    bias = torch.from_numpy((0.02 * rng.standard_normal(width)).astype(np.float32)).cuda()
    out = torch.zeros((rows, width), dtype=torch.int16, device="cuda")
    amax = torch.zeros(rows, dtype=torch.int32, device="cuda")
    int8.linear(a, sa, w, sw, bias, rows, width, kp, _capi.EPI_16, out, width, act=_capi.ACT_GELU,
                out_dtype=odt, row_amax=amax)
    kpo = (width + 15) // 16 * 16
    q = torch.full((rows, kpo), 9, dtype=torch.int8, device="cuda")
    s = torch.zeros(rows, device="cuda")
    int8.quantize_rows_amax(out, odt, rows, width, width, kpo, amax, q, s)
    torch.cuda.synchronize()
    hid = oracle.decode16(out.cpu().numpy().view(np.uint16), f16)
    oq, os_ = oracle.quantize_rows(hid, kp=kpo)
    assert (q.cpu().numpy() == oq).all()
    assert same_f32(s.cpu().numpy(), os_)


# ------------------------------------------------------------------ FFN blocks
def ref_weights(n):
    # crates/kata_nn/tests/int8_kernels.rs:352-357
    i = np.arange(n)
    return (((i * 7) % 61).astype(np.float32) / np.float32(123.0) - np.float32(0.25)).astype(np.float32)


@pytest.mark.parametrize("rows,mid,hidden", [(1, 512, 16), (1025, 512, 128), (1025, 512, 512), (1025, 512, 520),
                                             (1025, 512, 472), (3, 512, 1160), (3, 384, 1152), (3, 512, 1536)])
def test_swiglu_ffn_bit_exact(cuda, oracle, rows, mid, hidden):
    """int8_kernels.rs:329-431 shapes: fused FFN == unfused fp16-boundary composition."""
    torch = cuda
    i = np.arange(rows * mid)
    x = np.where(i < mid, 0.0, (i % 97).astype(np.float32) / np.float32(43.0) - 1).astype(np.float32)
    x16 = oracle.f16_encode(x.reshape(rows, mid))
    dual_w = ref_weights(2 * hidden * mid).reshape(2 * hidden, mid)
    down_w = ref_weights(mid * hidden).reshape(mid, hidden)
    dual = int8.Int8Weight(dual_w, _capi.LAYOUT_SWIGLU_DUAL)
    down = int8.Int8Weight(down_w)
    ws = int8.Int8Workspace(rows, max(mid, hidden), max(mid, hidden))
    res = torch.full((rows, mid), 0.125, device="cuda")
    ws.ffn(dev(torch, x16), dual, down, res, rows)
    torch.cuda.synchronize()
    ref, _ = oracle.swiglu_ffn_f16(oracle.decode16(x16, True), dual_w, down_w, np.full((rows, mid), 0.125, np.float32))
    assert same_f32(host(res), ref)


@pytest.mark.parametrize("rows,mid,hidden", [(1, 384, 1152), (361, 512, 16), (1025, 384, 472), (2888, 512, 1160)])
def test_swiglu_ffn_rms_bit_exact(cuda, oracle, rows, mid, hidden):
    """int8_kernels.rs:10-199 shapes: RMS -> quant -> FFN -> residual, bitwise."""
    torch = cuda
    x = rms_input(rows, mid)
    gamma = ((np.arange(mid) % 101).astype(np.float32) / np.float32(37.0) - 1).astype(np.float32)
    w = lambda n: (((np.arange(n) * 7) % 61).astype(np.float32) / np.float32(123.0) - np.float32(0.25)).astype(np.float32)
    dual_w = w(2 * hidden * mid).reshape(2 * hidden, mid)
    down_w = w(mid * hidden).reshape(mid, hidden)
    dual = int8.Int8Weight(dual_w, _capi.LAYOUT_SWIGLU_DUAL)
    down = int8.Int8Weight(down_w)
    ws = int8.Int8Workspace(rows, max(mid, hidden), max(mid, hidden))
    res = dev(torch, x)
    ws.ffn_rms(dev(torch, gamma), 1e-5, dual, down, res, rows)
    torch.cuda.synchronize()
    ref, _ = oracle.swiglu_ffn_f16(None, dual_w, down_w, x, rms=(gamma, 1e-5))
    assert same_f32(host(res), ref)


@pytest.mark.parametrize("rows,c,f", [(361, 768, 3072), (1000, 256, 1024), (23104, 768, 3072)])
def test_gelu_ffn_bit_exact(cuda, oracle, rows, c, f):
    """BASELINE config-2 block (bf16 residual, GELU), bitwise against the oracle."""
    torch = cuda
    rng = np.random.default_rng(rows + c + f)
    resid = oracle.bf16_encode(rng.standard_normal((rows, c)).astype(np.float32))
    gamma = (1 + 0.02 * rng.standard_normal(c)).astype(np.float32)
    up_w = (0.02 * rng.standard_normal((f, c))).astype(np.float32)
    down_w = (0.02 * rng.standard_normal((c, f))).astype(np.float32)
    up_b = (0.02 * rng.standard_normal(f)).astype(np.float32)
    down_b = (0.02 * rng.standard_normal(c)).astype(np.float32)
    up, down = int8.Int8Weight(up_w), int8.Int8Weight(down_w)
    ws = int8.Int8Workspace(rows, max(c, f), f)
    r = dev(torch, resid)
    ws.ffn_gelu_rms(dev(torch, gamma), 1e-6, up, dev(torch, up_b), down, dev(torch, down_b), r, rows)
    torch.cuda.synchronize()
    ref, _ = oracle.gelu_ffn_bf16(resid, gamma, 1e-6, up_w, up_b, down_w, down_b)
    got = host(r, np.uint16)
    assert (got == ref).all(), f"{(got != ref).sum()} of {got.size} differ"


# ------------------------------------------------------------------ bf16 GEMM
@pytest.mark.parametrize("m,n,k", [(361, 384, 768), (1000, 768, 208), (130, 96, 64), (4096, 2304, 768)])
def test_bf16_linear_matches_fp32(cuda, m, n, k):
    torch = cuda
    g = torch.Generator(device="cpu").manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w = (0.05 * torch.randn(n, k, generator=g)).to(torch.bfloat16).cuda()
    bias = (0.1 * torch.randn(n, generator=g)).cuda()
    out = torch.zeros(m, n, device="cuda")
    int8.bf16_linear(a, w, bias, m, n, k, _capi.EPI_F32, out, n)
    torch.cuda.synchronize()
    ref = a.float() @ w.float().T + bias
    err = (out - ref).abs().max().item()
    assert err <= 1e-4 * max(1.0, ref.abs().max().item()), err
    out16 = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    int8.bf16_linear(a, w, bias, m, n, k, _capi.EPI_16, out16, n, act=_capi.ACT_NONE)
    torch.cuda.synchronize()
    assert torch.equal(out16, out.to(torch.bfloat16))


@pytest.mark.parametrize("m,n,k,ldo", [(300, 136, 64, 140), (4096, 136, 768, 144), (361, 72, 48, 76)])
def test_f32_output_ragged_padded_rows(cuda, oracle, m, n, k, ldo):
    """fp32 outputs through the staging tiles and TMA stores with N not a
    multiple of 16 columns and a row stride above N: bitwise against the
    oracle (16-bit GEMM + bias; INT8 dequant), and the padding columns of
    every row keep their guard values."""
    torch = cuda
    rng = np.random.default_rng(m + n + k)
    guard = np.float32(-7.25)
    # 16-bit GEMM (binary16 operands) + bias
    a = oracle.f16_encode(rng.standard_normal((m, k)).astype(np.float32))
    w = oracle.f16_encode((0.05 * rng.standard_normal((n, k))).astype(np.float32))
    bias = (0.1 * rng.standard_normal(n)).astype(np.float32)
    out = torch.full((m, ldo), float(guard), device="cuda")
    int8.f16_linear(torch.from_numpy(a.view(np.int16)).cuda(), torch.from_numpy(w.view(np.int16)).cuda(),
                    torch.from_numpy(bias).cuda(), m, n, k, _capi.EPI_F32, out, ldo)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = (oracle.tc_gemm16(a, w, f16=True) + bias[None, :]).astype(np.float32)
    assert same_f32(got[:, :n], ref)
    assert (got[:, n:] == guard).all()
    # INT8 GEMM, fp32 dequant epilogue, no bias
    kp = (k + 15) // 16 * 16
    aq = rng.integers(-127, 128, (m, kp), dtype=np.int8)
    wq = rng.integers(-127, 128, (n, kp), dtype=np.int8)
    sa = (rng.random(m) * 0.01).astype(np.float32)
    sw = (rng.random(n) * 0.01).astype(np.float32)
    out2 = torch.full((m, ldo), float(guard), device="cuda")
    int8.linear(dev(torch, aq), torch.from_numpy(sa).cuda(), dev(torch, wq), torch.from_numpy(sw).cuda(), None,
                m, n, kp, _capi.EPI_F32, out2, ldo)
    torch.cuda.synchronize()
    got2 = out2.cpu().numpy()
    assert same_f32(got2[:, :n], oracle.dequant(oracle.igemm(aq, wq), sa, sw))
    assert (got2[:, n:] == guard).all()
