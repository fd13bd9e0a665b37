"""Pins the MXFP8 oracle (oracle/mxfp8.py) to the reference's own known
answers: the codec boundary tests of Rust_KataGo
crates/kata_nn/tests/test_mxfp8.rs:244-280 and the layout/padding test at
:282-314.  CPU only."""

import numpy as np

from oracle import mxfp8 as mx


def test_half_codec_known_answers():
    codes = np.arange(0x7C00, dtype=np.uint16)
    assert np.array_equal(mx.half_encode(mx.half_decode(codes)), codes)
    neg = codes | np.uint16(0x8000)
    assert np.array_equal(mx.half_encode(mx.half_decode(neg)), neg)
    assert mx.half_encode(1.00048828125) == 0x3C00
    assert mx.half_encode(1.00146484375) == 0x3C02
    assert mx.half_encode(2.0 ** -25) == 0
    assert mx.half_encode(mx.next_up(np.float32(2.0 ** -25))) == 1


def test_fp8_codebook_midpoints_and_saturation():
    assert mx.fp8_encode(np.float32(-0.0)) == 0x80
    assert mx.fp8_encode(np.float32(500.0)) == 0x7E
    assert mx.fp8_encode(np.float32(-500.0)) == 0xFE
    codes = np.arange(127)
    dec = mx.fp8_decode(codes)
    assert np.array_equal(mx.fp8_encode(dec.astype(np.float32)), codes)
    mid = ((dec[:-1] + dec[1:]) / 2).astype(np.float32)
    below = np.nextafter(mid, np.float32(-np.inf))
    above = np.nextafter(mid, np.float32(np.inf))
    assert np.array_equal(mx.fp8_encode(below), codes[:-1])
    assert np.array_equal(mx.fp8_encode(above), codes[:-1] + 1)
    even = np.where(codes[:-1] % 2 == 0, codes[:-1], codes[:-1] + 1)
    assert np.array_equal(mx.fp8_encode(mid), even)
    for bad in (np.nan, np.inf, -np.inf):
        try:
            mx.fp8_encode(np.float32(bad))
        except ValueError:
            continue
        raise AssertionError("non-finite must be rejected")


def test_scale_encode_powers():
    for e in (-127, -126, -120, -20, -1, 0, 1, 20, 120, 127):
        p = np.float32(2.0 ** e)
        assert mx.scale_encode(p) == e + 127
        assert mx.scale_encode(mx.next_up(p)) == min(e + 128, 254)


def test_layout_padding_and_source_precision():
    rows, k, stride = 129, 344, 357
    src = mx.test_input(rows, k, stride, 29, False, False)
    p = mx.quantize(src, rows, k, stride)
    assert p.status == 0
    assert np.all(p.values[:, k:] == 0)
    visited = np.zeros(p.scales.size, bool)
    for r in range(rows):
        for b in range(p.blocks):
            off = int(mx.packed_offset(r, b, p.blocks4))
            assert not visited[off]
            visited[off] = True
    assert np.all(p.scales[~visited] == 0)
    assert p.logical_scales[0, 0] == 127
    assert np.all(p.values[0, :32] == 0)
    edge = np.ones(32, np.float32)
    edge[0] = 448.0
    edge[1] = mx.next_up(np.float32(1.0625))
    rounded = mx.half_decode(mx.half_encode(edge))
    assert not np.array_equal(mx.quantize(edge, 1, 32, 32).values, mx.quantize(rounded, 1, 32, 32).values)


def test_nonfinite_block_semantics_and_weight_overflow():
    x = np.ones(64, np.float32)
    x[3] = np.nan
    x[40] = np.inf
    p = mx.quantize(x, 1, 64, 64)
    assert p.status == mx.STATUS_NAN | mx.STATUS_INF
    assert list(p.logical_scales[0]) == [127, 127]
    assert np.all(p.values == 0)
    w = np.zeros(64, np.float32)
    w[35] = np.finfo(np.float32).max
    assert mx.quantize(w, 1, 64, 64, check_weight=True).status & mx.STATUS_WEIGHT_OVERFLOW


def test_dyadic_reference_is_exact_in_fp32():
    w = mx.quantize(mx.test_input(24, 72, 85, 43, False, True), 24, 72, 85)
    x = mx.quantize(mx.test_input(17, 72, 79, 45, True, True), 17, 72, 79)
    exact, _ = mx.reference(w, x)
    assert np.array_equal(exact, exact.astype(np.float32).astype(np.float64))
