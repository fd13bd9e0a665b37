"""CPU oracle for the quantized trunk forward — TEST INFRASTRUCTURE ONLY.

The checker, never the product.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``) may import
this package.  It wraps ``kb_oracle.c`` — a plain-C restatement of the
reference's CPU arithmetic for the W8A8 path (Rust_KataGo, crates/kata_nn;
each C function cites the lines it follows) — plus numpy restatements of the
attention, MXFP8 codec and trunk pieces.

Parity of this oracle is pinned against the reference's own known answers and
closed-form test inputs in ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "kb_oracle.c"
LIB = HERE / "liboracle.so"

CFLAGS = ["-O3", "-fno-fast-math", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC", "-std=c11"]


def build() -> Path:
    """Compile kb_oracle.c with gcc (needs no GPU).  OpenMP is used when the
    compiler has it (it only parallelises independent rows)."""
    if LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    errors = []
    for cc in ("/usr/bin/gcc", os.environ.get("CC"), "gcc", "cc"):
        if not cc:
            continue
        for flags in (CFLAGS, [f for f in CFLAGS if f != "-fopenmp"]):
            res = subprocess.run([cc, *flags, str(SRC), "-o", str(tmp), "-lm"], capture_output=True, text=True)
            if res.returncode == 0:
                os.replace(tmp, LIB)
                return LIB
            errors.append(f"{cc} {' '.join(flags)}: {res.stderr.strip()[-300:]}")
    raise RuntimeError("cannot build the CPU oracle:\n" + "\n".join(errors))


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        P = ctypes.c_void_p
        I = ctypes.c_int
        F = ctypes.c_float
        Z = ctypes.c_size_t
        sig = {
            "or_f16_encode": (ctypes.c_uint16, [F]),
            "or_f16_decode": (F, [ctypes.c_uint16]),
            "or_bf16_encode": (ctypes.c_uint16, [F]),
            "or_bf16_decode": (F, [ctypes.c_uint16]),
            "or_encode16": (None, [P, Z, I, P]),
            "or_decode16": (None, [P, Z, I, P]),
            "or_silu_exp": (F, [F]),
            "or_silu": (F, [F]),
            "or_gelu": (F, [F]),
            "or_act": (None, [P, Z, I, P]),
            "or_int8_quantize_weights": (I, [P, I, I, P, P]),
            "or_int8_quantize_rows": (None, [P, I, I, I, I, P, P]),
            "or_int8_rms_quantize": (None, [P, I, I, I, P, F, I, I, P, P, P]),
            "or_igemm": (None, [P, P, I, I, I, P, I]),
            "or_dequant": (None, [P, P, P, I, I, P]),
            "or_dequant_bias": (None, [P, P, P, P, I, I, P]),
            "or_w8a8_project_half": (None, [P, I, I, P, P, I, I, P]),
            "or_max_threads": (I, []),
            "or_set_threads": (I, [I]),
            "or_attention_tc": (None, [P, I, I, I, I, F, I, P]),
            "or_tc_gemm16": (None, [P, P, I, I, I, I, P]),
            "or_rope_tables": (None, [P, I, I, P, P]),
            "or_tc_gemm_mxf8": (None, [P, P, P, P, I, I, I, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def padded16(k: int) -> int:
    return (k + 15) // 16 * 16


# ------------------------------------------------------------------ codecs
def f16_encode(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_encode16(_p(x), x.size, 1, _p(out))
    return out


def bf16_encode(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_encode16(_p(x), x.size, 0, _p(out))
    return out


def decode16(bits, f16: bool) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, np.float32)
    lib().or_decode16(_p(bits), bits.size, 1 if f16 else 0, _p(out))
    return out


def round16(x, f16: bool) -> np.ndarray:
    return decode16(f16_encode(x) if f16 else bf16_encode(x), f16)


def act(x, kind: int) -> np.ndarray:
    """kind: 0 none, 1 GELU (erf form), 2 SiLU; elementwise, same op order as the GPU."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().or_act(_p(x), x.size, kind, _p(out))
    return out


# ------------------------------------------------------------------ INT8 path
def quantize_weights(w: np.ndarray):
    """QuantizedWeights::new (int8.rs:171-211) -> (q [n, kp] int8, scales [n] f32)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    kp = padded16(k)
    q = np.zeros((n, kp), np.int8)
    s = np.zeros(n, np.float32)
    rc = lib().or_int8_quantize_weights(_p(w), n, k, _p(q), _p(s))
    if rc:
        raise ValueError(f"invalid INT8 weights (code {rc})")
    return q, s


def quantize_rows(x: np.ndarray, kp: int | None = None):
    """Per-token absmax quantisation of float rows (values already on a 16-bit grid)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, width = x.shape
    kp = kp or padded16(width)
    q = np.zeros((rows, kp), np.int8)
    s = np.zeros(rows, np.float32)
    lib().or_int8_quantize_rows(_p(x), rows, width, width, kp, _p(q), _p(s))
    return q, s


def rms_quantize(x: np.ndarray, gamma: np.ndarray, eps: float, f16: bool, kp: int | None = None):
    """Fused RMSNorm -> 16-bit boundary -> INT8 (int8_ops.cu:8-47). Returns (q, scales, normed)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    gamma = np.ascontiguousarray(gamma, dtype=np.float32)
    rows, width = x.shape
    kp = kp or padded16(width)
    q = np.zeros((rows, kp), np.int8)
    s = np.zeros(rows, np.float32)
    normed = np.zeros((rows, width), np.float32)
    lib().or_int8_rms_quantize(_p(x), rows, width, width, _p(gamma), eps, 1 if f16 else 0, kp, _p(q), _p(s), _p(normed))
    return q, s, normed


def igemm(a: np.ndarray, w: np.ndarray, threads: int = 0) -> np.ndarray:
    """int32 dots[m, n] = a[m, kp] . w[n, kp] (int8_kernels.rs:287-291)."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    m, kp = a.shape
    n = w.shape[0]
    assert w.shape[1] == kp
    out = np.zeros((m, n), np.int32)
    lib().or_igemm(_p(a), _p(w), m, n, kp, _p(out), threads)
    return out


def dequant_bias(dots: np.ndarray, sa: np.ndarray, sw: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """fma(f32(dot) * sa, sw, bias): the dequant plus bias of the BASELINE
    topology's projections, the bias added by one fused multiply-add."""
    dots = np.ascontiguousarray(dots, dtype=np.int32)
    m, n = dots.shape
    out = np.zeros((m, n), np.float32)
    lib().or_dequant_bias(_p(dots), _p(np.ascontiguousarray(sa, np.float32)), _p(np.ascontiguousarray(sw, np.float32)),
                          _p(np.ascontiguousarray(bias, np.float32)), m, n, _p(out))
    return out


def dequant(dots: np.ndarray, sa: np.ndarray, sw: np.ndarray) -> np.ndarray:
    """(f32(dot) * sa) * sw with two rounded multiplies (int8_ops.cu:182)."""
    dots = np.ascontiguousarray(dots, dtype=np.int32)
    m, n = dots.shape
    out = np.zeros((m, n), np.float32)
    lib().or_dequant(_p(dots), _p(np.ascontiguousarray(sa, np.float32)), _p(np.ascontiguousarray(sw, np.float32)), m, n, _p(out))
    return out


def w8a8_project_half(x16: np.ndarray, wq: np.ndarray, sw: np.ndarray, threads: int = 1) -> np.ndarray:
    """The reference's full CPU W8A8 projection (int8_kernels.rs:273-301) -> fp16 bits."""
    x16 = np.ascontiguousarray(x16, dtype=np.uint16)
    m, k = x16.shape
    n = wq.shape[0]
    out = np.zeros((m, n), np.uint16)
    lib().or_w8a8_project_half(_p(x16), m, k, _p(np.ascontiguousarray(wq)), _p(np.ascontiguousarray(sw, np.float32)), n, threads, _p(out))
    return out


def tc_gemm16(a_bits: np.ndarray, w_bits: np.ndarray, f16: bool = False) -> np.ndarray:
    """fp32 [m, n] = a[m, k] . w[n, k]^T with the tensor cores' accumulation
    (kb_oracle.c or_tc_gemm16) from 16-bit operand bits."""
    a_bits = np.ascontiguousarray(a_bits, np.uint16)
    w_bits = np.ascontiguousarray(w_bits, np.uint16)
    m, k = a_bits.shape
    n = w_bits.shape[0]
    assert w_bits.shape[1] == k
    out = np.empty((m, n), np.float32)
    lib().or_tc_gemm16(_p(a_bits), _p(w_bits), m, n, k, 1 if f16 else 0, _p(out))
    return out


def tc_gemm_mxf8(a, w) -> np.ndarray:
    """fp32 [m, n] accumulator of the block-scaled tensor-core GEMM of two
    MXFP8 operands (oracle.mxfp8.Packed: E4M3 codes and unpacked UE8M0 scales),
    with the tensor cores' accumulation (kb_oracle.c or_tc_gemm_mxf8)."""
    assert a.kp == w.kp
    ac = np.ascontiguousarray(a.values, np.uint8)
    wc = np.ascontiguousarray(w.values, np.uint8)
    asc = np.ascontiguousarray(a.logical_scales, np.uint8)
    wsc = np.ascontiguousarray(w.logical_scales, np.uint8)
    out = np.empty((a.rows, w.rows), np.float32)
    lib().or_tc_gemm_mxf8(_p(ac), _p(asc), _p(wc), _p(wsc), a.rows, w.rows, a.kp, _p(out))
    return out


def max_threads() -> int:
    return int(lib().or_max_threads())


def set_threads(threads: int) -> int:
    """OpenMP threads of the oracle's parallel loops; returns the count in effect."""
    return int(lib().or_set_threads(int(threads)))


# ------------------------------------------------------------------ composed FFN blocks
def swiglu_ffn_f16(x: np.ndarray, dual_w: np.ndarray, down_w: np.ndarray, residual: np.ndarray,
                   rms: tuple | None = None):
    """The reference's INT8 SwiGLU FFN with fp16 boundaries (int8.rs:1104-1259,
    int8_ops.cu:93-138, :187-194).

    x: fp16-grid input rows [rows, mid] (ignored when rms=(gamma, eps) is given:
    then the input is RMSNorm(residual) through int8_rms_quantize).
    dual_w: fp32 [2H, mid] = [gate; up]; down_w: fp32 [mid, H]; residual fp32 [rows, mid].
    Returns the new fp32 residual and intermediates.
    """
    dq, ds = quantize_weights(dual_w)
    wq, ws = quantize_weights(down_w)
    h = down_w.shape[1]
    if rms is not None:
        q, sa, _ = rms_quantize(residual, rms[0], rms[1], True, kp=dq.shape[1])
    else:
        q, sa = quantize_rows(x, kp=dq.shape[1])
    dots = igemm(q, dq)
    g = round16(dequant(dots[:, :h], sa, ds[:h]), True)
    u = round16(dequant(dots[:, h:], sa, ds[h:]), True)
    hidden = round16(u * act(g, 2), True)
    q2, s2 = quantize_rows(hidden, kp=wq.shape[1])
    dots2 = igemm(q2, wq)
    out = residual.astype(np.float32) + dequant(dots2, s2, ws)
    return out.astype(np.float32), {"q": q, "sa": sa, "hidden": hidden, "q2": q2, "s2": s2}


def gelu_ffn_bf16(residual_bf16: np.ndarray, gamma, eps, up_w, up_b, down_w, down_b, threads: int = 0):
    """BASELINE-topology FFN block on a bf16 residual: RMSNorm -> bf16 -> INT8 ->
    up GEMM (+bias) + GELU -> bf16 -> INT8 -> down GEMM (+bias) -> bf16 residual.
    residual_bf16: uint16 bits [rows, C].  Returns new residual bits and intermediates."""
    x = decode16(residual_bf16, False)
    uq, us = quantize_weights(up_w)
    dq, ds = quantize_weights(down_w)
    q, sa, normed = rms_quantize(x, gamma, eps, False, kp=uq.shape[1])
    dots = igemm(q, uq, threads)
    v = dequant(dots, sa, us) if up_b is None else dequant_bias(dots, sa, us, up_b)
    hidden = round16(act(v, 1), False)
    q2, s2 = quantize_rows(hidden, kp=dq.shape[1])
    dots2 = igemm(q2, dq, threads)
    d = dequant(dots2, s2, ds) if down_b is None else dequant_bias(dots2, s2, ds, down_b)
    out = bf16_encode((x + d).astype(np.float32))
    return out, {"q": q, "sa": sa, "hidden": hidden, "q2": q2, "s2": s2}
