"""CPU restatement of the nested (TF3) trunk forward — TEST INFRASTRUCTURE ONLY.

The reference lowers its native v17 TF3 model into a LayerGraph of
InitialConv (with the first block's pre_bn gate), per outer block a 768->384
Linear, pairs of RmsNorm / Attention (D = 32, RoPE) / RmsNorm / SwiGLU Ffn,
a GateSilu(384), a 384->768 Linear added to the raw trunk and the next
block's GateSilu(768), then TrunkFinal and the heads
(crates/kata_nn/src/native_model.rs:79-165); its CPU restatement of each layer
is crates/kata_nn/tests/debug_exec_units.rs:84-380 and its executor
crates/kata_nn/src/backends/cuda_exec.rs:1136-1700 (fp32 raw and inner
streams, fp16 at the 16-bit boundaries).

This module restates that graph with the product's arithmetic for each step:
  * binary16 tensor-core GEMMs (stem, the 768<->384 linears, unquantised
    attention projections, head linears) with the tensor cores' fp32
    accumulation (kb_oracle.c tc_block16, binary16 operands);
  * the INT8 projections and the SwiGLU FFN through the C oracle's bit-exact
    W8A8 restatements (rms_quantize with the fp16 boundary, igemm, dequant,
    swiglu_ffn_f16: int8.rs:171-211, int8_ops.cu:8-138, :187-194);
  * RoPE on the fp32 QKV projection, rounded to binary16 (native_model.rs:200-228);
  * attention with the kernel's definition (or_attention_tc, binary16 P) and
    the lowered graph's scale qk_scale^2 with qk_scale = 1/sqrt(sqrt(32));
  * the gates silu(x*scale + bias) with two rounded operations and the
    library's SiLU, rounded to binary16.
The weight blob is parsed independently of the product, from the layout
documented in include/katab200.h (KB_TOPO_NESTED).
"""

from __future__ import annotations

import numpy as np

from . import act, decode16, dequant, f16_encode, igemm, quantize_rows, quantize_weights, rms_quantize, round16, \
    swiglu_ffn_f16, tc_gemm16
from .trunk import SEQ, heads, rope_tables, rot, stem_inputs

HEAD_DIM = 32


def f16(x):
    """Round float32 values through binary16."""
    return round16(np.asarray(x, np.float32), True)


def gemm16(a, w):
    """fp32 a[m, k] . w[n, k]^T on the tensor cores with binary16 operands."""
    return tc_gemm16(f16_encode(np.asarray(a, np.float32)), f16_encode(np.asarray(w, np.float32)), f16=True)


def gate(x, scale, bias):
    """binary16(silu(x * scale + bias)): GateSilu / TrunkFinal (debug_exec_units.rs:254-282)."""
    v = ((np.asarray(x, np.float32) * scale[None, :]).astype(np.float32) + bias[None, :]).astype(np.float32)
    return f16(act(v, 2))


def attention_scale():
    """qk_scale^2 with qk_scale = 1 / sqrt(sqrt(32)) in fp32 (native_model.rs:195, cuda_exec.rs:1294)."""
    qk = np.float32(1.0) / np.sqrt(np.sqrt(np.float32(HEAD_DIM)))
    return float(np.float32(qk * qk))


def sections(c, nb, pairs, nh, m, h):
    secs = [("stem", (c, 217))]
    for i in range(nb):
        secs += [(f"{i}.pre_s", (c,)), (f"{i}.pre_b", (c,)), (f"{i}.pre_w", (m, c))]
        for j in range(pairs):
            p = f"{i}.{j}"
            secs += [(f"{p}.rms1", (m,)), (f"{p}.qkv", (3 * m, m)), (f"{p}.out", (m, m)),
                     (f"{p}.rope", (nh, HEAD_DIM // 2, 2)), (f"{p}.rms2", (m,)), (f"{p}.gate", (h, m)),
                     (f"{p}.up", (h, m)), (f"{p}.down", (m, h))]
        secs += [(f"{i}.post_s", (m,)), (f"{i}.post_b", (m,)), (f"{i}.post_w", (c, m))]
    secs += [("tip_g", (c,)), ("tip_b", (c,)), ("p1", (96, c)), ("g1", (96, c)), ("g1_b", (96,)),
             ("v1", (192, c)), ("v1_b", (192,)), ("gm", (96, 288)), ("pass1", (96, 288)), ("pass1_b", (96,)),
             ("pass2", (6, 96)), ("bias2", (96,)), ("conv2p", (6, 96)), ("v2", (192, 576)), ("v2_b", (192,)),
             ("value", (3, 192)), ("value_b", (3,)), ("misc", (10, 192)), ("misc_b", (10,)),
             ("moremisc", (8, 192)), ("moremisc_b", (8,)), ("own", (192,))]
    return secs


def parse(blob, topo):
    c, nb, pairs, nh, m, h = topo
    w, off = {}, 0
    for name, shape in sections(c, nb, pairs, nh, m, h):
        k = int(np.prod(shape))
        w[name] = np.asarray(blob[off:off + k], np.float32).reshape(shape)
        off += k
    if off != blob.size:
        raise ValueError("blob size does not match the nested topology")
    return w


def rope_qkv16(qkv32, cs, sn, n, nh):
    """Q and K rotated on the fp32 projection, then everything rounded to binary16."""
    c = nh * HEAD_DIM
    x = np.asarray(qkv32, np.float32).reshape(n, SEQ, 3, nh, HEAD_DIM).copy()
    x[:, :, 0] = rot(x[:, :, 0], cs, sn)
    x[:, :, 1] = rot(x[:, :, 1], cs, sn)
    return f16(x.reshape(n * SEQ, 3 * c))


def forward(blob, topo, spatial, glob, attn_int8=True, eps=1e-6, trace=False):
    """topo = (C, outer blocks, pairs per block, heads, mid, SwiGLU hidden).
    attn_int8: QKV and out projections in INT8 (else binary16, the reference's
    default Int8Scope::Ffn), or a pair (qkv_int8, out_int8).  Returns
    dict(policy, value, misc, moremisc, ownership) and, with trace, the
    binary16 planes kb_forward_trace records."""
    c, nb, pairs, nh, m, h = topo
    qkv_int8, out_int8 = attn_int8 if isinstance(attn_int8, tuple) else (attn_int8, attn_int8)
    w = parse(blob, topo)
    n = spatial.shape[0]
    scale = attention_scale()
    raw = gemm16(stem_inputs(spatial, glob), w["stem"])  # fp32 raw trunk
    planes = []
    for i in range(nb):
        g = gate(raw, w[f"{i}.pre_s"], w[f"{i}.pre_b"])
        planes.append(g)
        x = gemm16(g, w[f"{i}.pre_w"])  # fp32 inner stream
        for j in range(pairs):
            p = f"{i}.{j}"
            cs, sn = rope_tables(w[f"{p}.rope"])
            if qkv_int8:
                qw, qs = quantize_weights(w[f"{p}.qkv"])
                q, sa, _ = rms_quantize(x, w[f"{p}.rms1"], eps, True, kp=qw.shape[1])
                qkv32 = dequant(igemm(q, qw), sa, qs)
            else:
                _, _, normed = rms_quantize(x, w[f"{p}.rms1"], eps, True)
                qkv32 = gemm16(normed, w[f"{p}.qkv"])
            qkv = rope_qkv16(qkv32, cs, sn, n, nh)
            from .trunk import attention

            att = attention(qkv, None, None, n, nh, HEAD_DIM, rotate=False, scale=scale, f16=True)
            if out_int8:
                ow, os_ = quantize_weights(w[f"{p}.out"])
                q2, s2 = quantize_rows(att, kp=ow.shape[1])
                x = (x + dequant(igemm(q2, ow), s2, os_)).astype(np.float32)
            else:
                x = (x + gemm16(att, w[f"{p}.out"])).astype(np.float32)
            dual = np.concatenate([w[f"{p}.gate"], w[f"{p}.up"]], axis=0)
            x, _ = swiglu_ffn_f16(None, dual, w[f"{p}.down"], x, rms=(w[f"{p}.rms2"], eps))
        t = gate(x, w[f"{i}.post_s"], w[f"{i}.post_b"])
        raw = (raw + gemm16(t, w[f"{i}.post_w"])).astype(np.float32)
    g = gate(raw, w["tip_g"], w["tip_b"])
    planes += [g, g]
    wm = np.concatenate([w["p1"], w["g1"], w["v1"]], axis=0)
    bias = np.concatenate([np.zeros(96, np.float32), w["g1_b"], w["v1_b"]]).astype(np.float32)
    hp = (gemm16(g, wm) + bias[None, :]).astype(np.float32)
    out = heads(hp.reshape(n, SEQ, 384).astype(np.float64), w, n)
    if trace:
        out["trace"] = planes
    return out
