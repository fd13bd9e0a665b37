"""CPU restatement of the reference's MXFP8 arithmetic — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` (and the graft smoke/bench checkers) may import this module;
the product never does.  It restates, in numpy:

* the independent codecs of Rust_KataGo crates/kata_nn/tests/test_mxfp8.rs:8-130
  (IEEE half, the finite E4M3 codebook with ties to the even code, the UE8M0
  "smallest power of two >= amax/448" scale, the packed scale offset);
* the block-32 quantiser with the GPU kernel's status semantics
  (cuda-kernels/mxfp8.cu:36-79: a NaN/Inf element records a flag, its block
  gets scale 127 and zero bytes; a static FP32 weight whose decoded value
  overflows FP32 records WEIGHT_OVERFLOW);
* the exact fp64 reference on decoded operands and the gamma * sum|ab| error
  bound of test_mxfp8.rs:316-416;
* the deterministic test inputs of test_mxfp8.rs:191-239 (closed-form, so the
  reference's own cases are reproduced here without running it).

Pinned by the reference's known answers in tests/test_oracle_mxfp8.py.
"""

from __future__ import annotations

import numpy as np

STATUS_NAN, STATUS_INF, STATUS_OUTPUT_NONFINITE, STATUS_WEIGHT_OVERFLOW = 1, 2, 4, 8
MAX_K = 8192  # mxfp8.rs:31


# ---------------------------------------------------------------- IEEE half
def half_decode(bits) -> np.ndarray:
    """binary16 bits -> float32 (test_mxfp8.rs:8-22)."""
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


def half_encode(values) -> np.ndarray:
    """float32 -> binary16 bits, round to nearest even (test_mxfp8.rs:24-60);
    numpy's conversion is IEEE round-to-nearest-even, pinned by the known answers."""
    return np.asarray(values, np.float32).astype(np.float16).view(np.uint16)


# ---------------------------------------------------------------- E4M3 / UE8M0
def fp8_decode(codes) -> np.ndarray:
    """E4M3 byte -> float64 (test_mxfp8.rs:62-77); NaN (S.1111.111) is not decodable."""
    c = np.asarray(codes, np.int64)
    e, m = (c >> 3) & 15, c & 7
    if np.any((e == 15) & (m == 7)):
        raise ValueError("oracle cannot decode FP8 NaN")
    mag = np.where(e == 0, m * 2.0 ** -9, (8 + m) * np.exp2(e.astype(np.float64) - 10))
    return np.where(c & 128, -mag, mag)


_CODEBOOK = fp8_decode(np.arange(127))  # finite magnitudes, ascending with the code


def fp8_encode(values) -> np.ndarray:
    """Nearest finite E4M3 code, ties to the even code, sign kept (also for -0
    and values that round to zero) (test_mxfp8.rs:79-96).  Saturates at 448."""
    v = np.asarray(values, np.float32)
    if not np.all(np.isfinite(v)):
        raise ValueError("nonfinite input")
    mag = np.abs(v).astype(np.float64).ravel()
    hi = np.clip(np.searchsorted(_CODEBOOK, mag), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dl, dh = np.abs(_CODEBOOK[lo] - mag), np.abs(_CODEBOOK[hi] - mag)
    pick = np.where(dl < dh, lo, np.where(dh < dl, hi, np.where(lo % 2 == 0, lo, hi)))
    code = pick.astype(np.uint8).reshape(v.shape)
    return code | np.where(np.signbit(v), np.uint8(128), np.uint8(0))


def scale_encode(ratio) -> np.ndarray:
    """Smallest e in [-127, 127] with 2^e >= ratio, as the byte e + 127; 254 when
    none (test_mxfp8.rs:98-108).  ratio is the already rounded fp32 amax/448."""
    r = np.asarray(ratio, np.float32).astype(np.float64)
    if np.any(~np.isfinite(r)) or np.any(r < 0):
        raise ValueError("scale ratio must be finite and >= 0")
    mant, ex = np.frexp(r)  # r = mant * 2^ex, mant in [0.5, 1)
    e = np.where(mant == 0.5, ex - 1, ex)
    e = np.where(r == 0, -127, e)
    return (np.clip(e, -127, 127) + 127).astype(np.uint8)


def packed_offset(row, block, blocks4):
    """Byte offset of (row, 32-wide K block) in the packed scale layout:
    512-byte tiles of 128 rows x 4 blocks (test_mxfp8.rs:124-129, mxfp8.cu:75-77)."""
    row = np.asarray(row, np.int64)
    block = np.asarray(block, np.int64)
    return (((row // 128) * (blocks4 // 4) + block // 4) * 512 + (row % 32) * 16 + ((row % 128) // 32) * 4
            + block % 4)


def dimensions(rows: int, k: int):
    """(kp, blocks4, data_len, scale_len) (mxfp8.rs:56-76)."""
    if rows <= 0 or k <= 0 or k > MAX_K:
        raise ValueError(f"invalid MXFP8 dimensions rows={rows} K={k}")
    kp = -(-k // 32) * 32
    blocks4 = -(-(kp // 32) // 4) * 4
    return kp, blocks4, rows * kp, -(-rows // 128) * 128 * blocks4


class Packed:
    def __init__(self, rows, k):
        self.rows, self.k = rows, k
        self.kp, self.blocks4, n_data, n_scale = dimensions(rows, k)
        self.blocks = self.kp // 32
        self.values = np.zeros((rows, self.kp), np.uint8)
        self.logical_scales = np.zeros((rows, self.blocks), np.uint8)
        self.scales = np.zeros(n_scale, np.uint8)
        self.status = 0

    def decoded(self) -> np.ndarray:
        """float64 [rows, k] from the logical (unswizzled) scales (test_mxfp8.rs:178-190)."""
        v = fp8_decode(self.values[:, :self.k])
        s = np.repeat(self.logical_scales.astype(np.float64) - 127, 32, axis=1)[:, :self.k]
        return v * np.exp2(s)


def quantize(source, rows: int, k: int, stride: int, check_weight: bool = False) -> Packed:
    """Block-32 MXFP8 quantisation of float32 rows (test_mxfp8.rs:131-176) with
    the GPU kernel's handling of non-finite inputs (mxfp8.cu:47-65)."""
    src = np.asarray(source, np.float32).ravel()
    p = Packed(rows, k)
    x = np.zeros((rows, p.kp), np.float32)
    if stride == k:
        x[:, :k] = src[:rows * k].reshape(rows, k)
    else:
        for r in range(rows):
            x[r, :k] = src[r * stride:r * stride + k]
    nan, inf = np.isnan(x), np.isinf(x)
    if nan.any():
        p.status |= STATUS_NAN
    if inf.any():
        p.status |= STATUS_INF
    xb = x.reshape(rows, p.blocks, 32)
    bad = (nan | inf).reshape(rows, p.blocks, 32).any(axis=2)
    xb = np.where((nan | inf).reshape(xb.shape), np.float32(0), xb)
    amax = np.abs(xb).max(axis=2)
    zero = (amax == 0) | bad
    ratio = np.where(zero, np.float32(1), amax / np.float32(448.0)).astype(np.float32)
    scale = np.where(zero, np.uint8(127), scale_encode(ratio)).astype(np.uint8)
    scaled = (xb.astype(np.float64) * np.exp2(127.0 - scale.astype(np.float64))[:, :, None]).astype(np.float32)
    codes = fp8_encode(scaled)
    codes = np.where(zero[:, :, None], np.uint8(0), codes).reshape(rows, p.kp)
    codes[:, k:] = 0
    p.values[:] = codes
    p.logical_scales[:] = scale
    rr, bb = np.meshgrid(np.arange(rows), np.arange(p.blocks), indexing="ij")
    p.scales[packed_offset(rr, bb, p.blocks4).ravel()] = scale.ravel()
    if check_weight:
        dec = fp8_decode(codes.reshape(rows, p.blocks, 32)) * np.exp2(scale.astype(np.float64) - 127)[:, :, None]
        if np.any(np.abs(dec) > np.finfo(np.float32).max):
            p.status |= STATUS_WEIGHT_OVERFLOW
    return p


# ---------------------------------------------------------------- references
def reference(weight: Packed, activation: Packed, residual=None):
    """(exact [rows, n] float64, sum_abs [rows, n]) of decoded operands
    (test_mxfp8.rs:316-366): sum_k w*x (+ residual) and sum_k |w*x| (+ |r|)."""
    w, x = weight.decoded(), activation.decoded()
    exact = x @ w.T
    sum_abs = np.abs(x) @ np.abs(w).T
    if residual is not None:
        r = np.asarray(residual, np.float64).reshape(exact.shape)
        exact = exact + r
        sum_abs = sum_abs + np.abs(r)
    return exact, sum_abs


def gamma(k: int) -> float:
    """gamma_(k+2) for fp32 accumulation plus the fp64 reference (test_mxfp8.rs:378-383)."""
    ops = k + 2
    u, du = 2.0 ** -24, 2.0 ** -53
    return ops * u / (1 - ops * u) + ops * du / (1 - ops * du)


def next_up(v):
    v = np.float32(v)
    return np.nextafter(v, np.float32(np.inf))


def next_down(v):
    v = np.float32(v)
    return np.nextafter(v, np.float32(-np.inf))


def check_output(actual, half: bool, k: int, exact, sum_abs, bitwise: bool):
    """Raises AssertionError unless every output is bit-identical to the rounded
    exact value (dyadic cases) or inside exact +- gamma*sum_abs, widened to the
    neighbouring half values for half outputs (test_mxfp8.rs:370-416)."""
    exact = np.asarray(exact, np.float64).ravel()
    if half:
        bits = np.asarray(actual, np.uint16).ravel()
        val = half_decode(bits).astype(np.float64)
    else:
        bits = np.asarray(actual, np.float32).ravel().view(np.uint32)
        val = bits.view(np.float32).astype(np.float64)
    assert np.all(np.isfinite(val)), "non-finite output"
    if bitwise:
        exp = half_encode(exact.astype(np.float32)) if half else exact.astype(np.float32).view(np.uint32)
        bad = np.nonzero(bits != exp)[0]
        assert bad.size == 0, f"dyadic bitwise mismatch at {bad[:8]} got {bits[bad[:8]]} want {exp[bad[:8]]}"
        return 0.0
    bound = gamma(k) * np.asarray(sum_abs, np.float64).ravel()
    low, high = exact - bound, exact + bound
    if half:
        low = half_decode(half_encode(np.nextafter(low.astype(np.float32), np.float32(-np.inf)))).astype(np.float64)
        high = half_decode(half_encode(np.nextafter(high.astype(np.float32), np.float32(np.inf)))).astype(np.float64)
    bad = np.nonzero((val < low) | (val > high))[0]
    assert bad.size == 0, f"outside the fp64 bound at {bad[:8]}: {val[bad[:8]]} vs {exact[bad[:8]]}"
    return float(np.max(np.abs(val - exact))) if val.size else 0.0


# ---------------------------------------------------------------- test inputs
def _mix(v):
    v = np.asarray(v, np.uint64) & 0xFFFFFFFF
    v ^= v >> 16
    v = (v * 0x7FEB352D) & 0xFFFFFFFF
    v ^= v >> 15
    v = (v * 0x846CA68B) & 0xFFFFFFFF
    return v ^ (v >> 16)


def test_input(rows: int, k: int, stride: int, seed: int, half: bool, exact: bool) -> np.ndarray:
    """The reference's closed-form operand generator (test_mxfp8.rs:200-239):
    float32 [rows * stride], NaN in the stride padding, zeros / negative zeros
    in row 0's first block, optionally pre-rounded through half."""
    out = np.full(rows * stride, np.nan, np.float32)
    r = np.arange(rows, dtype=np.uint64)[:, None]
    c = np.arange(k, dtype=np.uint64)[None, :]
    m32 = 0xFFFFFFFF
    noise = _mix((seed + r * 65537 + c * 257) & m32)
    blk = c // 32
    if exact:
        expo = (_mix((seed ^ r ^ blk) & m32) % 4).astype(np.int64) - 4
        frac = (noise % 9).astype(np.float32) - np.float32(4.0)
    else:
        expo = (_mix((seed ^ ((r * 131) & m32) ^ ((blk * 977) & m32)) & m32) % 13).astype(np.int64) - 8
        frac = ((noise % 20001).astype(np.int64) - 10000).astype(np.float32) / np.float32(10000.0)
    val = (frac * np.exp2(expo.astype(np.float32))).astype(np.float32)
    val = np.broadcast_to(val, (rows, k)).copy()
    if rows > 0:
        n0 = min(k, 32)
        val[0, :n0] = np.where(np.arange(n0) % 2 == 0, np.float32(0.0), np.float32(-0.0))
    if half:
        val = half_decode(half_encode(val))
    out.reshape(rows, stride)[:, :k] = val
    return out
