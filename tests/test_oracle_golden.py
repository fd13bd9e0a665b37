"""CPU tests: pin the C oracle to the reference's own known answers and to the
independent closed-form fixture in tests/golden/ (no GPU needed)."""

import math
import struct

import numpy as np
import pytest

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "int8_dot_cases.npz"


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bits_f32(b):
    return struct.unpack("<f", struct.pack("<I", b))[0]


def next_up(x):
    return bits_f32(f32_bits(x) + 1) if x > 0 else (bits_f32(1) if x == 0 else -bits_f32(f32_bits(-x) - 1))


def test_weight_quant_known_answers(oracle):
    # crates/kata_nn/tests/int8_kernels.rs:201-222
    w = np.zeros((4, 8), np.float32)
    w[1] = [127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, -127.0]
    w[2] = 0.001
    w[3] = -2.0
    q, s = oracle.quantize_weights(w)
    assert q.shape == (4, 16)
    assert s[0] == 1.0
    assert list(q[1, :8]) == [127, 0, 2, 2, 0, -2, -2, -127]
    assert list(q[2, :8]) == [127] * 8
    assert (q[:, 8:] == 0).all()
    w[0, 0] = np.nan
    with pytest.raises(ValueError):
        oracle.quantize_weights(w)
    with pytest.raises(ValueError):
        oracle.quantize_weights(np.zeros((3, 8), np.float32))  # N % 4 != 0


def test_half_codec_known_answers(oracle):
    # crates/kata_nn/tests/test_mxfp8.rs:245-256
    lib = oracle.lib()
    codes = np.arange(0x7C00, dtype=np.uint16)
    for c in (codes, codes | 0x8000):
        dec = oracle.decode16(c, True)
        assert (oracle.f16_encode(dec) == c).all()
    assert lib.or_f16_encode(1.00048828125) == 0x3C00
    assert lib.or_f16_encode(1.00146484375) == 0x3C02
    assert lib.or_f16_encode(2.0 ** -25) == 0
    assert lib.or_f16_encode(next_up(2.0 ** -25)) == 1
    # agrees with numpy's IEEE float16 rounding on a dense sweep
    x = np.random.default_rng(1).standard_normal(200000).astype(np.float32) * 300
    assert (oracle.f16_encode(x) == x.astype(np.float16).view(np.uint16)).all()


def test_bf16_codec(oracle):
    x = np.random.default_rng(2).standard_normal(100000).astype(np.float32)
    b = oracle.bf16_encode(x)
    # RNE: decoding is within half an ulp, ties to even
    d = oracle.decode16(b, False)
    ulp = np.abs(d).view(np.uint32).astype(np.int64)
    assert np.all(np.abs(d.astype(np.float64) - x) <= 2.0 ** (np.floor(np.log2(np.abs(x) + 1e-30)) - 8) + 1e-38)
    assert oracle.lib().or_bf16_encode(1.00390625) == 0x3F80  # tie -> even
    assert oracle.lib().or_bf16_encode(1.01171875) == 0x3F82  # tie -> even (up)
    del ulp


@pytest.mark.parametrize("shape", [tuple(s) for s in np.load(GOLDEN)["shapes"]])
def test_int8_dot_cases_match_fixture(oracle, shape):
    """The oracle reproduces the closed-form cases of int8_kernels.rs:224-327 bit for bit."""
    rows, n, k = shape
    g = np.load(GOLDEN)
    key = f"{rows}_{n}_{k}_"
    wq, ws = oracle.quantize_weights(g[key + "w"])
    assert (wq == g[key + "wq"]).all() and (ws.view(np.uint32) == g[key + "ws"].view(np.uint32)).all()
    x = oracle.decode16(g[key + "x16"], True)[:, :k]
    q, sa = oracle.quantize_rows(np.ascontiguousarray(x), kp=wq.shape[1])
    assert (q[:, :k] == g[key + "q"]).all() and (q[:, k:] == 0).all()
    assert (sa.view(np.uint32) == g[key + "sa"].view(np.uint32)).all()
    dots = oracle.igemm(q, wq)
    assert (dots == g[key + "dots"]).all()
    val = oracle.dequant(dots, sa, ws)
    assert (oracle.f16_encode(val) == g[key + "half"]).all()
    assert ((g[key + "initial"] + val).view(np.uint32) == g[key + "residual"].view(np.uint32)).all()


def test_reference_cpu_projection_matches_composition(oracle):
    g = np.load(GOLDEN)
    rows, n, k = 65, 72, 48
    key = f"{rows}_{n}_{k}_"
    x16 = np.ascontiguousarray(g[key + "x16"][:, :k])
    out = oracle.w8a8_project_half(x16, g[key + "wq"], g[key + "ws"], threads=2)
    assert (out == g[key + "half"]).all()


def test_silu_exp_accuracy(oracle):
    """The SiLU's e^x: accurate on [-20, 88.72], and 1 + e^x unchanged by its clamp."""
    lib = oracle.lib()
    xs = np.concatenate([np.linspace(-20, 88.72, 20001), np.random.default_rng(3).uniform(-20, 20, 20000)])
    worst = 0.0
    for x in xs.astype(np.float32):
        got = lib.or_silu_exp(float(x))
        ref = math.exp(float(x))
        worst = max(worst, abs(got - ref) / ref)
    assert worst < 3e-7  # about 2.5 ulp worst case, typically < 1 ulp
    # every float above ln(FLT_MAX) overflows, the largest below it does not
    top = np.float32(88.72283)
    assert math.isfinite(lib.or_silu_exp(float(np.nextafter(top, np.float32(0)))))
    for x in (np.nextafter(np.float32(88.72284), np.float32(100)), 88.75, 89.0, 1e4, math.inf):
        assert lib.or_silu_exp(float(x)) == math.inf
    # below the clamp, 1 + e^x rounds to 1 as the clamped value's does
    for x in (-17.4, -20.0, -50.0, -1e4, -math.inf):
        assert np.float32(1) + np.float32(lib.or_silu_exp(float(x))) == np.float32(1)
    # a NaN argument reaches the SiLU division, which returns NaN
    assert math.isnan(lib.or_silu(float("nan")))
    assert lib.or_silu(-1e4) == 0.0 and math.copysign(1, lib.or_silu(-1e4)) == -1
    assert lib.or_silu(1e4) == 1e4


def test_silu_every_binary16_input(oracle):
    """SiLU of every finite binary16 value against float64 with the fp32
    denominator (which overflows to inf for g < -88.72, as expf's does), to
    2 ulp of fp32."""
    lib = oracle.lib()
    h = np.arange(1 << 16, dtype=np.uint16).view(np.float16)
    h = h[np.isfinite(h)].astype(np.float32)
    with np.errstate(over="ignore"):
        for g in h:
            got = np.float32(lib.or_silu(float(g)))
            d = np.float32(1.0 + math.exp(-float(g))) if g > -700 else np.float32(np.inf)
            ref = float(g) / float(d)
            assert abs(got - ref) <= 2.5e-7 * abs(ref) + 1e-44, (g, got, ref)


def test_gelu_silu_accuracy(oracle):
    lib = oracle.lib()
    xs = np.linspace(-12, 12, 40001).astype(np.float32)
    gelu_err = max(abs(lib.or_gelu(float(x)) - 0.5 * x * (1 + math.erf(x / math.sqrt(2)))) / max(1.0, abs(x))
                   for x in xs)
    assert gelu_err < 3.5e-5  # clamp of Phi at |x| = 4 dominates (3.2e-5)
    assert lib.or_gelu(0.0) == 0.0 and lib.or_gelu(100.0) == 100.0 and lib.or_gelu(-100.0) == 0.0
    silu_err = max(abs(lib.or_silu(float(x)) - x / (1 + math.exp(-x))) / max(1e-3, abs(x)) for x in xs)
    assert silu_err < 1e-6


def rms_rows(rows, mid):
    # crates/kata_nn/tests/int8_kernels.rs:21-33
    i = np.arange(rows * mid)
    v = ((i * 127 + i // mid) % 997).astype(np.float32) / np.float32(191.0) - np.float32(2.5)
    kind = (i // mid) % 7
    v = np.where(kind == 0, 0.0, np.where(kind == 1, v * np.float32(1e-18), np.where(kind == 2, v * np.float32(1e12), v)))
    return v.astype(np.float32).reshape(rows, mid)


@pytest.mark.parametrize("rows,mid", [(1, 384), (361, 512), (1025, 384)])
def test_rms_quantize_semantics(oracle, rows, mid):
    """RMS quantiser: float64 restatement within rounding, exact special rows."""
    x = rms_rows(rows, mid)
    x[0, 0] = np.inf
    if rows > 1:
        x[1, 0] = np.nan
    gamma = ((np.arange(mid) % 101).astype(np.float32) / np.float32(37.0) - 1).astype(np.float32)
    q, s, normed = oracle.rms_quantize(x, gamma, 1e-5, True)
    assert np.isnan(s[0]) and (q[0] == 0).all()
    if rows > 1:
        assert np.isnan(s[1]) and (q[1] == 0).all()
    for r in range(2, rows):
        xr = x[r].astype(np.float64)
        rstd = 1.0 / math.sqrt((xr * xr).sum() / mid + 1e-5)
        v = (xr * rstd * gamma).astype(np.float16).astype(np.float64)
        amax = np.abs(v).max()
        if amax == 0:
            assert s[r] == 1.0 and (q[r] == 0).all()
            continue
        assert abs(s[r] - amax / 127) <= 2e-3 * amax / 127  # fp16 grid may shift amax by 1 ulp
        ref_q = np.clip(np.rint(v / (amax / 127)), -127, 127)
        assert np.abs(q[r, :mid].astype(np.int64) - ref_q).max() <= 1
