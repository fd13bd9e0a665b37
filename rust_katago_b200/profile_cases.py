"""Kernel cases for profiling the library under Nsight Compute.

    python -m rust_katago_b200.profile_cases <case> [batch]

Each case runs one kernel family at the b11c768 trunk's batch-256 shapes (or
one whole forward) twice, so `ncu -s 1 -c 1` captures a warm launch:

  trunk   two forwards without a graph (104 kernels each)
  tf3     two forwards of the nested TF3 b11c768 trunk (INT8 recipe) without a graph
  tf3ffn  the same with the FFN-scope recipe (binary16 QKV and out projections)
  up      INT8 GEMM 92416x3072x768 + bias + GELU (the FFN up projection)
  down    INT8 GEMM 92416x768x3072 + bias + bf16 residual
  out     INT8 GEMM 92416x768x768 + bias + bf16 residual (the attention out-projection)
  attn    attention, 256 positions x 12 heads x 64 (Q and K already rotated, the trunk's path)
  attn32  attention of the TF3 trunk: 256 positions x 12 heads x 32, binary16
  qkv     INT8 GEMM 92416x2304x768 with the rotary epilogue (the trunk's QKV projection)
  quant   streaming quantiser of the 92416x3072 bf16 FFN hidden
  rms     fused RMSNorm -> bf16 -> INT8 quantiser, 92416x768
  mxup    MXFP8 block-scaled GEMM 92416x3072x768 -> bf16 (the up projection)
  swiglu  INT8 SwiGLU FFN of the TF3 trunk, 92416 rows, mid 384, hidden 1152: dual GEMM
          (92416x2304x384, SwiGLU epilogue) -> requantiser -> down GEMM + fp32 residual
  mxquant MXFP8 block-32 quantiser of a 92416x768 bf16 activation
  decode  output decoding + post-processing of 256 positions (kb_decode_device, legality mask)
"""

from __future__ import annotations

import sys


def main(argv):
    import torch

    from . import _capi, backend, int8, synthetic

    case = argv[1] if len(argv) > 1 else "trunk"
    batch = int(argv[2]) if len(argv) > 2 else 256
    m = batch * 361
    torch.cuda.set_device(0)
    if case in ("trunk", "tf3", "tf3ffn"):
        topo = {"trunk": synthetic.B11C768, "tf3": synthetic.TF3_B11C768,
                "tf3ffn": synthetic.TF3_B11C768_FFN}[case]
        model = backend.CudaBackend.load_model(topo, synthetic.make_blob(topo, 1234))
        h = backend.CudaBackend.create_compute_handle(model, batch)
        sp, gl = synthetic.make_positions(batch, 5)
        dsp, dgl = torch.from_numpy(sp).cuda(), torch.from_numpy(gl).cuda()
        dout = torch.zeros(batch * backend.OUT_PER_POS, device="cuda")
        for _ in range(2):
            h.forward_device(batch, dsp, dgl, dout, use_graph=False)
    elif case in ("up", "down", "qkv", "out"):
        n, k, epi, act = {"up": (3072, 768, _capi.EPI_16, _capi.ACT_GELU),
                          "down": (768, 3072, _capi.EPI_RES16, 0),
                          "out": (768, 768, _capi.EPI_RES16, 0),
                          "qkv": (2304, 768, _capi.EPI_16, 0)}[case]
        # (the qkv case times the plain 16-bit epilogue; the trunk adds the rotary tables)
        a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda")
        w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda")
        sa = torch.rand(m, device="cuda") * 0.01
        sw = torch.rand(n, device="cuda") * 0.01
        b = torch.rand(n, device="cuda")
        out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        for _ in range(2):
            int8.linear(a, sa, w, sw, b, m, n, k, epi, out, n, act=act)
    elif case in ("attn", "attn32"):
        heads, d = 12, 64 if case == "attn" else 32
        dt, tdt = (_capi.DT_BF16, torch.bfloat16) if case == "attn" else (_capi.DT_F16, torch.float16)
        qkv = torch.randn(m, 3 * heads * d, device="cuda").to(tdt)
        out = torch.empty(m, heads * d, dtype=tdt, device="cuda")
        for _ in range(2):
            _capi.call("kb_attention", qkv.data_ptr(), 0, 0, out.data_ptr(), batch, heads,
                       d, d ** -0.5, dt, int(torch.cuda.current_stream().cuda_stream))
    elif case == "quant":
        x = torch.randn(m, 3072, device="cuda").to(torch.bfloat16).view(torch.int16)
        amax = torch.full((m,), 0x41000000, dtype=torch.int32, device="cuda")  # |x| <= 8.0 as f32 bits
        q = torch.empty(m, 3072, dtype=torch.int8, device="cuda")
        s = torch.empty(m, device="cuda")
        for _ in range(2):
            int8.quantize_rows_amax(x, _capi.DT_BF16, m, 3072, 3072, 3072, amax, q, s)
    elif case == "rms":
        x = torch.randn(m, 768, device="cuda").to(torch.bfloat16).view(torch.int16)
        g = torch.ones(768, device="cuda")
        q = torch.empty(m, 768, dtype=torch.int8, device="cuda")
        s = torch.empty(m, device="cuda")
        for _ in range(2):
            int8.rms_quantize(x, _capi.DT_BF16, m, 768, 768, g, 1e-6, _capi.DT_BF16, 768, q, s)
    elif case == "decode":
        import numpy as np

        rng = np.random.default_rng(0)
        raw = torch.from_numpy(rng.standard_normal(batch * backend.OUT_PER_POS).astype(np.float32)).cuda()
        rows = backend.row_params(batch, symmetry=rng.integers(0, 8, batch), policy_optimism=0.3)
        d_rows = torch.from_numpy(np.ascontiguousarray(rows).view(np.uint8).reshape(batch, 24)).cuda()
        legal = torch.from_numpy((rng.random((batch, 362)) < 0.8).astype(np.uint8)).cuda()
        out = torch.empty(batch * backend.DEC_PER_POS, device="cuda")
        for _ in range(2):
            backend.decode_device(batch, raw, d_rows, legal, out, int(torch.cuda.current_stream().cuda_stream))
    elif case == "swiglu":
        import numpy as np

        mid, hid = 384, 1152
        rng = np.random.default_rng(0)
        dual = int8.Int8Weight((0.05 * rng.standard_normal((2 * hid, mid))).astype(np.float32),
                               _capi.LAYOUT_SWIGLU_DUAL)
        down = int8.Int8Weight((0.05 * rng.standard_normal((mid, hid))).astype(np.float32))
        ws = int8.Int8Workspace(m, hid, hid)
        x = torch.randn(m, mid, device="cuda").to(torch.float16).view(torch.int16)
        res = torch.zeros(m, mid, device="cuda")
        for _ in range(2):
            ws.ffn(x, dual, down, res, m)
    elif case in ("mxup", "mxquant"):
        import numpy as np

        from . import mxfp8

        k, n = 768, 3072
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        _, _, data, scale = mxfp8.dimensions(m, k)
        q = torch.empty(data, dtype=torch.uint8, device="cuda")
        sc = torch.empty(scale, dtype=torch.uint8, device="cuda")
        st = torch.zeros(2, dtype=torch.int32, device="cuda")
        mxfp8.reset_status(st)
        if case == "mxquant":
            for _ in range(2):
                mxfp8.quantize(x, _capi.DT_BF16, m, k, k, q, sc, st)
        else:
            w = mxfp8.Mxfp8Weight(np.random.default_rng(0).standard_normal((n, k), np.float32) * 0.02, n, k, k)
            mxfp8.quantize(x, _capi.DT_BF16, m, k, k, q, sc, st)
            out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
            for _ in range(2):
                mxfp8.gemm(q, sc, m, w, out, n, mxfp8.OUT_BF16, st)
    else:
        raise SystemExit(f"unknown case {case!r}; see the module docstring")
    torch.cuda.synchronize()
    print("ok", case, batch)


if __name__ == "__main__":
    main(sys.argv)
