"""CPU restatement of the full trunk forward — TEST INFRASTRUCTURE ONLY.

Follows the reference's CPU restatement of every LayerGraph layer
(Rust_KataGo crates/kata_nn/tests/debug_exec_units.rs:84-380) on the
BASELINE b11c768 topology, with the INT8 linears through the C oracle
(quantize_weights / rms_quantize / quantize_rows / igemm / dequant, bit-exact
restatements of the reference's W8A8 arithmetic) and the same 16-bit rounding
points as the product: bf16 residual stream, bf16 QKV / attention output /
FFN hidden, bf16-rounded stem and head weights.

The 16-bit and MXFP8 tensor-core GEMMs (stem, head linears, bf16 and
block-scaled projections) and the attention kernel's q.k and P.V products
follow the tensor cores' own fp32 accumulation (kb_oracle.c tc_block16: blocks of 16 products aligned to the
largest exponent, truncated, rounded toward zero), and the attention softmax
the kernel's definition (two key halves with their own maxima, P rounded to
bf16 for P.V, the kernel's polynomial 2^x; kb_oracle.c or_attention_tc), so
the residual stream is reproduced bit for bit.  The policy/value heads after
the head linears are computed in float64 (their fp32 order is not restated)
and compared with a tolerance.

The weight blob is parsed here independently of the product's parser, from
the layout documented in include/katab200.h (kb_model_blob_floats).
"""

from __future__ import annotations

import math

import numpy as np

from . import (bf16_encode, decode16, dequant, dequant_bias, igemm, quantize_rows, quantize_weights, rms_quantize,
               round16, tc_gemm16)

SEQ, SIDE = 361, 19
EPS = 1e-6


def _sections(c, nb, nh, hd, f):
    secs = [("stem", (c, 217))]
    for i in range(nb):
        secs += [(f"{i}.rms1", (c,)), (f"{i}.qkv", (3 * c, c)), (f"{i}.out", (c, c)), (f"{i}.rms2", (c,)),
                 (f"{i}.up", (f, c)), (f"{i}.up_b", (f,)), (f"{i}.down", (c, f)), (f"{i}.down_b", (c,)),
                 (f"{i}.rope", (nh, hd // 2, 2))]
    secs += [("tip_g", (c,)), ("tip_b", (c,)), ("p1", (96, c)), ("g1", (96, c)), ("g1_b", (96,)),
             ("v1", (192, c)), ("v1_b", (192,)), ("gm", (96, 288)), ("pass1", (96, 288)), ("pass1_b", (96,)),
             ("pass2", (6, 96)), ("bias2", (96,)), ("conv2p", (6, 96)), ("v2", (192, 576)), ("v2_b", (192,)),
             ("value", (3, 192)), ("value_b", (3,)), ("misc", (10, 192)), ("misc_b", (10,)),
             ("moremisc", (8, 192)), ("moremisc_b", (8,)), ("own", (192,))]
    return secs


def parse(blob, c, nb, nh, hd, f):
    w, off = {}, 0
    for name, shape in _sections(c, nb, nh, hd, f):
        k = int(np.prod(shape))
        w[name] = np.asarray(blob[off:off + k], np.float32).reshape(shape)
        off += k
    if off != blob.size:
        raise ValueError("blob size does not match the topology")
    return w


def bf(x):
    """Round float32 values through bf16."""
    return round16(np.asarray(x, np.float32), False)


def silu64(x):
    return x / (1.0 + np.exp(-x))


def stem_inputs(spatial, glob):
    """[n*361, 217]: 3x3 taps (ic*9 + ky*3 + kx, zero padded) then 19 globals (debug_exec_units.rs:101-129)."""
    n = spatial.shape[0]
    pad = np.zeros((n, 22, SIDE + 2, SIDE + 2), np.float32)
    pad[:, :, 1:-1, 1:-1] = spatial
    taps = np.zeros((n, SIDE, SIDE, 22, 3, 3), np.float32)
    for ky in range(3):
        for kx in range(3):
            taps[:, :, :, :, ky, kx] = pad[:, :, ky:ky + SIDE, kx:kx + SIDE].transpose(0, 2, 3, 1)
    a = np.concatenate([taps.reshape(n, SEQ, 22 * 9), np.repeat(glob[:, None, :], SEQ, axis=1)], axis=2)
    return a.reshape(n * SEQ, 217)


def rope_tables(freqs):
    """cos/sin [361, heads, pairs]: angle = x*f0 + y*f1 in float32, then the C
    library's cosf / sinf, as the reference's f32::cos / f32::sin compute them
    (native_model.rs:200-228; kb_oracle.c or_rope_tables)."""
    from . import lib

    freqs = np.ascontiguousarray(freqs, np.float32)
    nh, pairs, _ = freqs.shape
    cs = np.zeros((SEQ, nh, pairs), np.float32)
    sn = np.zeros_like(cs)
    lib().or_rope_tables(freqs.ctypes.data, nh, pairs, cs.ctypes.data, sn.ctypes.data)
    return cs, sn


def rot(t, cs, sn):
    """RoPE of interleaved pairs (2p, 2p+1) in float32 with each product and sum
    rounded: (x c - y s, x s + y c); t [n, 361, heads, hd], tables [361, heads, hd/2]."""
    t = np.asarray(t, np.float32)
    a, b = t[..., 0::2], t[..., 1::2]
    ra = (a * cs[None]).astype(np.float32) - (b * sn[None]).astype(np.float32)
    rb = (a * sn[None]).astype(np.float32) + (b * cs[None]).astype(np.float32)
    out = np.empty_like(t)
    out[..., 0::2] = ra
    out[..., 1::2] = rb
    return out


def rope_qkv(qkv32, cs, sn, n, nh, hd):
    """The QKV projection's epilogue: Q and K rotated on the fp32 projection,
    then everything rounded to bf16 (rotary tables native_model.rs:200-228)."""
    c = nh * hd
    x = np.asarray(qkv32, np.float32).reshape(n, SEQ, 3, nh, hd).copy()
    x[:, :, 0] = rot(x[:, :, 0], cs, sn)
    x[:, :, 1] = rot(x[:, :, 1], cs, sn)
    return bf(x.reshape(n * SEQ, 3 * c))


def attention_scale(hd):
    """The trunk's softmax scale, fp32(1 / fp32(sqrt(hd)))."""
    return float(np.float32(1.0) / np.sqrt(np.float32(hd)))


def attention(qkv, cs, sn, n, nh, hd, rotate=True, exact=False, scale=None, f16=False):
    """Softmax attention per (position, head) (debug_exec_units.rs:161-242).
    rotate: apply RoPE to the 16-bit Q and K here and round to bf16 (the
    attention kernel's own rotation); False when Q and K arrive rotated.

    exact=False (default): the attention kernel's own definition of the
    softmax, restated in C (kb_oracle.c or_attention_tc: two key halves with
    their own maxima, P rounded to bf16 for P.V, row sums of the unrounded P,
    the kernel's 2^x), so that only fp32 summation order separates it from
    the kernel.  exact=True: softmax in float64 with P unrounded (the
    mathematical definition; the reference kernel keeps P in fp16).  f16: the
    16-bit type is binary16 (qkv values on its grid), else bfloat16."""
    c = nh * hd
    x = np.asarray(qkv, np.float32).reshape(n, SEQ, 3, nh, hd)
    q, k, v = x[:, :, 0], x[:, :, 1], x[:, :, 2]
    if rotate:
        q, k = bf(rot(q, cs, sn)), bf(rot(k, cs, sn))
    if scale is None:
        scale = attention_scale(hd)
    if not exact:
        from . import f16_encode, lib

        packed = np.ascontiguousarray(np.stack([q, k, v], axis=2).reshape(n * SEQ, 3 * c), np.float32)
        bits = np.ascontiguousarray(f16_encode(packed) if f16 else bf16_encode(packed))
        out = np.empty((n * SEQ, c), np.uint16)
        lib().or_attention_tc(bits.ctypes.data, n, SEQ, nh, hd, np.float32(scale), 1 if f16 else 0, out.ctypes.data)
        return decode16(out, f16)
    q, k = q.astype(np.float64), k.astype(np.float64)
    v = v.astype(np.float64)
    s = np.einsum("bqhd,bkhd->bhqk", q, k) * float(scale)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhqk,bkhd->bqhd", p, v)
    return round16(o.reshape(n * SEQ, c).astype(np.float32), f16)


def _mx_weight(w):
    """An MXFP8 weight (E4M3 codes + UE8M0 scales) quantised from the original fp32."""
    from . import mxfp8 as mx

    n, k = w.shape
    return mx.quantize(w, n, k, k, check_weight=True)


def _mx_linear(xv, wq):
    """fp32 accumulator of an MXFP8 projection: the activation's 16-bit values
    quantised block-32 (mxfp8.cu:36-79), then the block-scaled GEMM with the
    tensor cores' accumulation (kb_oracle.c or_tc_gemm_mxf8)."""
    from . import mxfp8 as mx, tc_gemm_mxf8

    rows, k = xv.shape
    return tc_gemm_mxf8(mx.quantize(np.ascontiguousarray(xv, np.float32), rows, k, k), wq)


def _project(kind, src, wmat, bias=None, gamma=None):
    """fp32 result (bias included) of one trunk projection of bf16 rows `src`
    in precision `kind` ("int8", "mxfp8" or "bf16"), with the pre-norm RMSNorm
    fused when `gamma` is given — the single-precision branches of forward()
    per projection: INT8 quantises the (normalised) 16-bit rows per token and
    dequantises exactly, MXFP8 quantises them block-32, bf16 multiplies the
    16-bit values by the bf16-rounded weight with the tensor cores' fp32
    accumulation (tc_gemm16)."""
    if kind == "int8":
        qw, qs = quantize_weights(wmat)
        if gamma is not None:
            q, sa, _ = rms_quantize(src, gamma, EPS, False, kp=qw.shape[1])
        else:
            q, sa = quantize_rows(src, kp=qw.shape[1])
        dots = igemm(q, qw)
        return dequant(dots, sa, qs) if bias is None else dequant_bias(dots, sa, qs, bias)
    xv = rms_quantize(src, gamma, EPS, False)[2] if gamma is not None else src
    if kind == "mxfp8":
        acc = _mx_linear(xv, _mx_weight(wmat))
    elif kind == "bf16":
        acc = tc_gemm16(bf16_encode(xv), bf16_encode(wmat))
    else:
        raise ValueError(f"unknown projection precision {kind!r}")
    return acc if bias is None else (acc + bias[None, :]).astype(np.float32)


def forward(blob, topo, spatial, glob, teacher=None, precision="int8"):
    """Returns dict(policy [n,6,362], value [n,3], misc [n,10], moremisc [n,8],
    ownership [n,361], residual [n*361, C]).

    precision "mxfp8" runs every trunk projection as the MXFP8 path does
    (block-32 E4M3 activations and weights, UE8M0 scales, fp32 accumulation);
    a 4-tuple of "int8" / "mxfp8" / "bf16" gives each projection (qkv, out,
    ffn_up, ffn_down) its own precision, as a precision recipe does.

    teacher: optional (stem [n*361, C], [attention [n*361, C] per block]) float
    arrays that replace the oracle's own stem GEMM and attention results — the
    two steps whose fp32 accumulation order cannot be reproduced on the CPU —
    so that every other step can be compared bit for bit.  With None in place
    of the attention list only the stem is replaced."""
    c, nb, nh, hd, f = topo
    w = parse(blob, c, nb, nh, hd, f)
    n = spatial.shape[0]
    if teacher is not None:
        x = np.asarray(teacher[0], np.float32)
    else:
        x = stem_output(blob, topo, spatial, glob)
    from . import act

    for i in range(nb):
        cs, sn = rope_tables(w[f"{i}.rope"])
        if isinstance(precision, (tuple, list)):
            pq, po, pu, pd = precision
            qkv = rope_qkv(_project(pq, x, w[f"{i}.qkv"], gamma=w[f"{i}.rms1"]), cs, sn, n, nh, hd)
            att = (attention(qkv, cs, sn, n, nh, hd, rotate=False) if teacher is None or teacher[1] is None
                   else np.asarray(teacher[1][i], np.float32))
            x = bf((x + _project(po, att, w[f"{i}.out"])).astype(np.float32))
            v = _project(pu, x, w[f"{i}.up"], bias=w[f"{i}.up_b"], gamma=w[f"{i}.rms2"])
            hidden = bf(act(v, 1))
            d = _project(pd, hidden, w[f"{i}.down"], bias=w[f"{i}.down_b"])
            x = bf((x + d).astype(np.float32))
            continue
        if precision == "mxfp8":
            wq, wo, wu, wd = (_mx_weight(w[f"{i}.{nm}"]) for nm in ("qkv", "out", "up", "down"))
            _, _, normed = rms_quantize(x, w[f"{i}.rms1"], EPS, False)
            qkv = rope_qkv(_mx_linear(normed, wq), cs, sn, n, nh, hd)
            att = (attention(qkv, cs, sn, n, nh, hd, rotate=False) if teacher is None or teacher[1] is None
                   else np.asarray(teacher[1][i], np.float32))
            x = bf((x + _mx_linear(att, wo)).astype(np.float32))
            _, _, normed = rms_quantize(x, w[f"{i}.rms2"], EPS, False)
            v = (_mx_linear(normed, wu) + w[f"{i}.up_b"][None, :]).astype(np.float32)
            hidden = bf(act(v, 1))
            d = (_mx_linear(hidden, wd) + w[f"{i}.down_b"][None, :]).astype(np.float32)
            x = bf((x + d).astype(np.float32))
            continue
        qw, qs = quantize_weights(w[f"{i}.qkv"])
        ow, os_ = quantize_weights(w[f"{i}.out"])
        uw, us = quantize_weights(w[f"{i}.up"])
        dw, ds = quantize_weights(w[f"{i}.down"])
        q, sa, _ = rms_quantize(x, w[f"{i}.rms1"], EPS, False, kp=qw.shape[1])
        qkv = rope_qkv(dequant(igemm(q, qw), sa, qs), cs, sn, n, nh, hd)
        att = (attention(qkv, cs, sn, n, nh, hd, rotate=False) if teacher is None or teacher[1] is None
               else np.asarray(teacher[1][i], np.float32))
        q2, s2 = quantize_rows(att, kp=ow.shape[1])
        x = bf((x + dequant(igemm(q2, ow), s2, os_)).astype(np.float32))
        q3, s3, _ = rms_quantize(x, w[f"{i}.rms2"], EPS, False, kp=uw.shape[1])
        v = dequant_bias(igemm(q3, uw), s3, us, w[f"{i}.up_b"])
        hidden = bf(act(v, 1))
        q4, s4 = quantize_rows(hidden, kp=dw.shape[1])
        d = dequant_bias(igemm(q4, dw), s4, ds, w[f"{i}.down_b"])
        x = bf((x + d).astype(np.float32))
    # trunk tip: silu(x*gamma + beta) (debug_exec_units.rs:272-282)
    g = bf(act(((x * w["tip_g"][None, :]).astype(np.float32) + w["tip_b"][None, :]).astype(np.float32), 2))
    out = heads(head_linears(g, w).reshape(n, SEQ, 384).astype(np.float64), w, n)
    out["residual"] = x
    return out


def heads(hp, w, n):
    """PolicyHead / ValueHead (debug_exec_units.rs:283-380) in float64."""
    p1, g1, v1 = hp[..., :96], hp[..., 96:192], hp[..., 192:]
    ga = silu64(g1)
    mean = ga.mean(axis=1)
    pooled = np.concatenate([mean, mean * 0.5, ga.max(axis=1)], axis=1)  # [n, 288]
    pass1 = silu64(pooled @ w["pass1"].T.astype(np.float64) + w["pass1_b"])
    pass2 = pass1 @ w["pass2"].T.astype(np.float64)  # [n, 6]
    gproj = pooled @ w["gm"].T.astype(np.float64) + w["bias2"]
    pa = silu64(p1 + gproj[:, None, :])
    moves = pa @ w["conv2p"].T.astype(np.float64)  # [n, 361, 6]
    policy = np.zeros((n, 6, 362))
    policy[:, :, :361] = moves.transpose(0, 2, 1)
    policy[:, :, 361] = pass2
    va = silu64(v1)
    vm = va.mean(axis=1)
    pooled_v = np.concatenate([vm, vm * 0.5, vm * 0.15], axis=1)  # [n, 576]
    hid = silu64(pooled_v @ w["v2"].T.astype(np.float64) + w["v2_b"])
    value = hid @ w["value"].T.astype(np.float64) + w["value_b"]
    misc = hid @ w["misc"].T.astype(np.float64) + w["misc_b"]
    more = hid @ w["moremisc"].T.astype(np.float64) + w["moremisc_b"]
    own = va @ w["own"].astype(np.float64)
    return {"policy": policy, "value": value, "misc": misc, "moremisc": more, "ownership": own}


def stem_output(blob, topo, spatial, glob):
    """The stem (3x3 conv + global linear as one bf16 GEMM on the tensor
    cores): bf16 values [n*361, C]."""
    w = parse(blob, *topo)
    return bf(tc_gemm16(bf16_encode(stem_inputs(spatial, glob)), bf16_encode(w["stem"])))


def head_linears(g, w):
    """fp32 [rows, 384] = g . [p1 | g1 | v1]^T on the tensor cores (bf16
    operands) + [0 | g1_b | v1_b], the biases added in fp32."""
    wm = np.concatenate([w["p1"], w["g1"], w["v1"]], axis=0)
    bias = np.concatenate([np.zeros(96, np.float32), w["g1_b"], w["v1_b"]]).astype(np.float32)
    return (tc_gemm16(bf16_encode(g), bf16_encode(wm)) + bias[None, :]).astype(np.float32)


def perturbed_stem_forward(blob, topo, spatial, glob, fraction=1e-4, seed=0, precision="int8"):
    """forward() with the stem output perturbed by one bf16 ulp (last mantissa
    bit flipped) on a seeded `fraction` of its elements: the smallest
    difference two correct implementations can have.  How far the outputs
    move measures the trunk's own sensitivity to last-bit differences."""
    from . import bf16_encode

    stem = stem_output(blob, topo, spatial, glob)
    bits = bf16_encode(stem)
    mask = np.random.default_rng(seed).random(bits.shape) < fraction
    bits = bits.copy()
    bits[mask] ^= 1
    return forward(blob, topo, spatial, glob, teacher=(decode16(bits, False), None), precision=precision)
