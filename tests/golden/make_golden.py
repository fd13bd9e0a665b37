"""Generate tests/golden/int8_dot_cases.npz — the reference's closed-form INT8
projection cases, evaluated by an implementation independent of oracle/.

Source of the cases: Rust_KataGo crates/kata_nn/tests/int8_kernels.rs:224-327
(`integer_dot_products_pruned_tails_and_dynamic_graph_scales`).  Its inputs are
closed-form formulas and its expected values are the test's own CPU formula:

    x      = f16(row == 0 ? 0 : ((row*13 + col*7) % 113) / 19 - 3)      (:234-241)
    w[i]   = i < k ? 0 : ((i*17 + i/k) % 127) / 127 - 0.5                 (:242-250)
    scale  = max|x| / 127 (1 for a zero row)                              (:273-276)
    q      = clamp(round_ties_even(x / scale), +-127)                     (:277-280)
    dot    = sum q * wq  (int32)                                          (:287-291)
    half   = f16((f32(dot) * scale) * w_scale)                            (:296-297)
    res    = initial + (f32(dot) * scale) * w_scale, initial=(i%17)/13    (:298-301)

Weights are quantised per output channel as QuantizedWeights::new
(src/backends/int8.rs:171-211).  Everything here is numpy (IEEE float32 ops,
numpy's own float16 rounding), not the C oracle, so the oracle is checked
against a second, independent restatement.  Run: python tests/golden/make_golden.py
"""

from pathlib import Path

import numpy as np

SHAPES = [(1, 16, 8), (3, 48, 24), (65, 72, 48), (1025, 48, 24), (3, 944, 512), (2, 512, 472),
          (3, 1536, 512), (4, 2304, 384)]
OUT = Path(__file__).resolve().parent / "int8_dot_cases.npz"


def f32(x):
    return np.float32(x)


def weight_quant(w: np.ndarray):
    n, k = w.shape
    kp = (k + 15) // 16 * 16
    q = np.zeros((n, kp), np.int8)
    s = np.zeros(n, np.float32)
    for r in range(n):
        amax = np.max(np.abs(w[r])).astype(np.float32)
        scale = f32(1.0) if amax == 0 else max(f32(amax / f32(127.0)), np.finfo(np.float32).tiny)
        s[r] = scale
        q[r, :k] = np.clip(np.rint((w[r] / scale).astype(np.float32)), -127, 127).astype(np.int8)
    return q, s


def case(rows, n, k):
    stride = (k + 15) // 16 * 16
    x = np.zeros((rows, k), np.float32)
    for row in range(1, rows):
        col = np.arange(k)
        x[row] = (((row * 13 + col * 7) % 113).astype(np.float32) / f32(19.0)) - f32(3.0)
    x16 = x.astype(np.float16)
    idx = np.arange(n * k)
    w = np.where(idx < k, f32(0.0), (((idx * 17 + idx // k) % 127).astype(np.float32) / f32(127.0)) - f32(0.5))
    w = w.astype(np.float32).reshape(n, k)
    wq, ws = weight_quant(w)
    xv = x16.astype(np.float32)
    amax = np.max(np.abs(xv), axis=1)
    scale = np.where(amax == 0, f32(1.0), (amax / f32(127.0)).astype(np.float32)).astype(np.float32)
    q = np.clip(np.rint((xv / scale[:, None]).astype(np.float32)), -127, 127).astype(np.int64)
    dots = (q @ wq[:, :k].astype(np.int64).T).astype(np.int32)
    expected = ((dots.astype(np.float32) * scale[:, None]).astype(np.float32) * ws[None, :]).astype(np.float32)
    half = expected.astype(np.float16).view(np.uint16)
    initial = ((np.arange(rows * n) % 17).astype(np.float32) / f32(13.0)).reshape(rows, n)
    residual = (initial + expected).astype(np.float32)
    xin = np.full((rows, stride), np.float16(31.0), np.float16)  # padding columns hold 31 (:232)
    xin[:, :k] = x16
    return {
        "x16": xin.view(np.uint16), "w": w, "wq": wq, "ws": ws, "q": q.astype(np.int8), "sa": scale,
        "dots": dots, "half": half, "initial": initial, "residual": residual,
    }


def main():
    arrays = {}
    for rows, n, k in SHAPES:
        c = case(rows, n, k)
        for name, val in c.items():
            arrays[f"{rows}_{n}_{k}_{name}"] = val
    arrays["shapes"] = np.array(SHAPES, np.int32)
    np.savez_compressed(OUT, **arrays)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
