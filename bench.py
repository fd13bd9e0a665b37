#!/usr/bin/env python
"""Benchmark of the quantized b11c768 trunk forward on B200 (positions/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload ...]

One process per GPU (torchrun for N > 1).  Positions are independent, so the
batch is sharded across ranks with no collective on the data path ("weak"
scaling: every rank runs the same per-GPU batch); the only collectives are the
barrier and the max-over-ranks reduction of the device time.

Timing: W untimed warm-up steps; K timed steps, each bracketed by its own CUDA
events on the launching stream, with an L2 flush (a 256 MiB write) between
steps outside the events; barrier + synchronize on both sides of the region;
the reported step time is the max over ranks.  ``e2e`` repeats the step through
the public API with pinned host buffers, the H2D copy of the step's inputs and
the D2H copy of its outputs inside the timed region.

``--impl reference`` times the reference's CPU arithmetic for the same workload
(the CPU oracle under oracle/, a restatement of the reference's quantized CPU
path: Rust_KataGo cannot be built in this image) on all host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "positions/sec b11c768 W8A8 fwd @1/2/4/8 B200; INT8 GEMM % tensor peak"
L2_FLUSH_BYTES = 256 << 20


# ncu summaries (profiles/*.md) of the kernels that can dominate the step.
PROFILE_OF_GEMM = {"up 768->3072 + GELU": "gemm_i8_up_gelu_b256.md", "attention": "attention_b256.md"}


def profile_traffic(gemm_label):
    """DRAM bytes (read + write) per launch recorded in the committed ncu summary, or None."""
    name = PROFILE_OF_GEMM.get(gemm_label)
    path = Path(__file__).resolve().parent / "profiles" / name if name else None
    if path is None or not path.exists():
        return None
    total = 0.0
    for key in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
        m = re.search(re.escape(key) + r"\s*\|\s*([0-9.]+)\s*MB", path.read_text())
        if not m:
            return None
        total += float(m.group(1)) * 1e6
    return total


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ workloads
class FfnWorkload:
    """one b11c768 FFN block at batch B (B*361 tokens).

    RMSNorm -> per-token INT8 quant -> W8A8 768->3072 GEMM + bias + GELU ->
    bf16 -> quant -> W8A8 3072->768 GEMM + bias + residual, on a bf16 residual
    stream.  Weights N(0, 0.02) int8 per channel, residual N(0, 1)."""

    name = "config2: one b11c768 FFN block (RMSNorm, W8A8 768->3072 GELU, W8A8 3072->768 + residual)"
    e2e_how = ("public API (Int8Workspace.ffn_gelu_rms on the residual copied in from pinned host memory and "
               "copied back each step)")

    def __init__(self, batch: int, torch, seed: int = 1234, build_device: bool = True):
        self.torch = torch
        self.batch = batch
        self.rows = batch * 361
        self.c, self.f = 768, 3072
        rng = np.random.default_rng(seed)
        self.gamma_h = (1 + 0.02 * rng.standard_normal(self.c)).astype(np.float32)
        self.up_w = (0.02 * rng.standard_normal((self.f, self.c))).astype(np.float32)
        self.down_w = (0.02 * rng.standard_normal((self.c, self.f))).astype(np.float32)
        self.up_b_h = (0.02 * rng.standard_normal(self.f)).astype(np.float32)
        self.down_b_h = (0.02 * rng.standard_normal(self.c)).astype(np.float32)
        x = rng.standard_normal((self.rows, self.c)).astype(np.float32)
        import oracle

        self.resid_h = oracle.bf16_encode(x) if not build_device else None
        if not build_device:
            return
        from rust_katago_b200 import int8

        self.resid_h = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        self.up = int8.Int8Weight(self.up_w)
        self.down = int8.Int8Weight(self.down_w)
        self.ws = int8.Int8Workspace(self.rows, self.f, self.f)
        self.gamma = torch.from_numpy(self.gamma_h).cuda()
        self.up_b = torch.from_numpy(self.up_b_h).cuda()
        self.down_b = torch.from_numpy(self.down_b_h).cuda()
        self.resid = torch.from_numpy(self.resid_h.view(np.int16)).cuda()
        self.pinned_in = torch.from_numpy(self.resid_h.view(np.int16)).pin_memory()
        self.pinned_out = torch.empty_like(self.pinned_in).pin_memory()
        self.stream = torch.cuda.current_stream()
        self.launches_per_step = 4

    @property
    def units_per_step(self):
        return self.batch

    def step(self):
        self.ws.ffn_gelu_rms(self.gamma, 1e-6, self.up, self.up_b, self.down, self.down_b, self.resid, self.rows)

    def e2e_run(self, steps: int):
        for _ in range(steps):
            self.resid.copy_(self.pinned_in, non_blocking=True)
            self.step()
            self.pinned_out.copy_(self.resid, non_blocking=True)
            self.torch.cuda.current_stream().synchronize()

    def e2e_bytes(self):
        b = self.rows * self.c * 2
        return b, b

    def gemms(self):
        from rust_katago_b200 import _capi

        return [("up 768->3072 + GELU", self.rows, self.f, self.c, _capi.EPI_16, _capi.ACT_GELU, 1),
                ("down 3072->768 + residual", self.rows, self.c, self.f, _capi.EPI_RES16, 0, 1)]

    def cpu_reference(self, positions: int, threads: int):
        """The CPU oracle on `positions` positions; returns seconds."""
        import oracle

        rows = positions * 361
        t0 = time.perf_counter()
        oracle.gelu_ffn_bf16(np.ascontiguousarray(self.resid_h[:rows]), self.gamma_h, 1e-6, self.up_w, self.up_b_h,
                             self.down_w, self.down_b_h, threads=threads)
        return time.perf_counter() - t0


def gemm_launcher(torch, m, n, k, epi, act):
    """A launch of the INT8 GEMM kernel on random operands of the given shape;
    the GELU projection also emits the row |max| as the trunk's launch does
    (the atomics feed its streaming requantiser)."""
    from rust_katago_b200 import _capi, int8

    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda")
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda")
    sa = torch.rand(m, device="cuda") * 0.01
    sw = torch.rand(n, device="cuda") * 0.01
    bias = torch.rand(n, device="cuda") * 0.01
    out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    amax = torch.zeros(m, dtype=torch.int32, device="cuda") if act == _capi.ACT_GELU else None

    def launch():
        int8.linear(a, sa, w, sw, bias, m, n, k, epi, out, n, act=act, row_amax=amax)

    return launch


class TrunkWorkload:
    """the full b11c768 W8A8 trunk forward at batch B per GPU.

    Stem (3x3 conv 22->768 + global linear, bf16 GEMM) -> 11 x [RMSNorm ->
    INT8 QKV -> RoPE attention 12x64 -> INT8 out-proj + residual -> RMSNorm ->
    INT8 768->3072 + GELU -> INT8 3072->768 + residual] -> trunk tip -> policy
    [B,6,362] / value [B,3] / misc / moremisc / ownership heads.  Synthetic
    seeded weights N(0,0.02) and positions (22 binary planes p=0.3, 19 global
    N(0,1)); one CUDA graph per forward."""

    name = "config3: full b11c768 W8A8 trunk forward (11 blocks, 12x64 attention, FFN 768->3072->768, heads)"
    e2e_how = ("public API (kb_submit_rows with a random board symmetry per row, applied on the device, and the "
               "outputs decoded on the device as the reference's finish_output decodes them / kb_finish_rows: "
               "pinned staging, H2D on the copy stream, graph, decode, D2H of the decoded rows, status check; "
               "the handle's two pipeline slots in use, batch k+1 submitted before batch k is finished)")
    dtype = "int8"
    kernel = "gemm_kernel<i8,256>"
    precision = "int8"

    def topology(self):
        from rust_katago_b200 import synthetic

        return synthetic.B11C768

    def __init__(self, batch: int, torch, seed: int = 1234, build_device: bool = True, rank: int = 0):
        from rust_katago_b200 import backend, synthetic

        self.torch = torch
        self.batch = batch
        self.topo = self.topology()
        self.blob = synthetic.make_blob(self.topo, seed)  # replicated weights: same seed on every rank
        # each rank evaluates its own shard of distinct positions
        self.spatial, self.glob = synthetic.make_positions(max(batch, 4), seed + 1 + 7919 * rank)
        if not build_device:
            return
        self.spatial, self.glob = self.spatial[:batch], self.glob[:batch]
        # one random board symmetry per row, as MCTS submits them (applied on the device)
        self.symmetry = np.random.default_rng(seed + 3 + rank).integers(0, 8, batch).astype(np.int32)
        # decoded on the device as the reference's finish_output decodes on the host
        self.rows = backend.row_params(batch, symmetry=self.symmetry)
        self.model = backend.CudaBackend.load_model(self.topo, self.blob, torch.cuda.current_device())
        self.handle = backend.CudaBackend.create_compute_handle(self.model, batch)
        self.d_spatial = torch.from_numpy(self.spatial).cuda()
        self.d_global = torch.from_numpy(self.glob).cuda()
        self.d_out = torch.zeros(batch * backend.OUT_PER_POS, device="cuda")
        self.stream = torch.cuda.ExternalStream(self.handle.stream)
        self.launches_per_step = 2 + 9 * self.topo.num_blocks + 3
        self.handle.warmup([batch])

    @property
    def units_per_step(self):
        return self.batch

    def step(self):
        self.handle.forward_device(self.batch, self.d_spatial, self.d_global, self.d_out, use_graph=True)

    def e2e_run(self, steps: int):
        """`steps` batches through kb_submit_rows / kb_finish_rows with the
        handle's two pipeline slots in use, as an evaluator thread drives it
        (cuda.rs keeps two in flight): batch k+1 is submitted before batch k is
        finished, so its host staging and input copies overlap batch k's
        forward; every batch's copies and decoded outputs are in the region."""
        tok = self.handle.submit_rows(self.spatial, self.glob, self.rows)
        for _ in range(steps - 1):
            nxt = self.handle.submit_rows(self.spatial, self.glob, self.rows)
            self.handle.finish_rows(tok)
            tok = nxt
        self.handle.finish_rows(tok)

    def e2e_bytes(self):
        from rust_katago_b200 import backend

        return (self.spatial.nbytes + self.glob.nbytes + self.symmetry.nbytes + self.rows.nbytes,
                self.batch * backend.DEC_PER_POS * 4 + 8)

    def gemms(self):
        """The trunk's INT8 GEMM shapes: (label, m, n, k, epilogue, act, launches per forward)."""
        from rust_katago_b200 import _capi

        m, c, f = self.batch * 361, 768, 3072
        nb = self.topo.num_blocks
        return [("qkv 768->2304", m, 3 * c, c, _capi.EPI_16, 0, nb),
                ("out 768->768 + residual", m, c, c, _capi.EPI_RES16, 0, nb),
                ("up 768->3072 + GELU", m, f, c, _capi.EPI_16, _capi.ACT_GELU, nb),
                ("down 3072->768 + residual", m, c, f, _capi.EPI_RES16, 0, nb)]

    def cpu_reference(self, positions: int, threads: int):
        import oracle.trunk as ot

        t = self.topo
        t0 = time.perf_counter()
        ot.forward(self.blob, (t.trunk_channels, t.num_blocks, t.num_heads, t.head_dim, t.ffn_channels),
                   self.spatial[:positions], self.glob[:positions], precision=self.precision)
        return time.perf_counter() - t0

    def gemm_launcher(self, m, n, k, epi, act):
        return gemm_launcher(self.torch, m, n, k, epi, act)

    def attention(self):
        """The trunk's attention launch (Q and K already rotated by the QKV
        epilogue, 12 heads x 64, bf16, row |max| for the next quantiser):
        (label, launcher, launches per forward, algorithmic bytes, FLOPs)."""
        from rust_katago_b200 import _capi

        torch, t = self.torch, self.topo
        m, c = self.batch * 361, t.trunk_channels
        qkv = (torch.randn(m, 3 * c, device="cuda") * 1.5).to(torch.bfloat16)
        out = torch.empty(m, c, dtype=torch.bfloat16, device="cuda")
        amax = torch.zeros(m, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream()

        def launch():
            _capi.call("kb_attention_amax", qkv.data_ptr(), out.data_ptr(), amax.data_ptr(), self.batch,
                       t.num_heads, t.head_dim, t.head_dim ** -0.5, _capi.DT_BF16, int(stream.cuda_stream))

        launch.keep = (qkv, out, amax)
        flops = 4.0 * 361 * 361 * t.head_dim * t.num_heads * self.batch
        return ("attention 12x64 (pre-rotated, row amax)", launch, t.num_blocks, 4 * m * c * 2, flops)


class TrunkMxfp8Workload(TrunkWorkload):
    """the same trunk with every projection MXFP8 (E4M3
    operands, UE8M0 scale per 32 K, fp32 accumulation on tcgen05
    kind::mxf8f6f4.block_scale); same seeds, weights quantised from fp32."""

    name = "config4: full b11c768 MXFP8 trunk forward (11 blocks, 12x64 attention, FFN 768->3072->768, heads)"
    dtype = "e4m3"
    kernel = "gemm_kernel<mxf8f6f4.block_scale,128>"
    precision = "mxfp8"

    def topology(self):
        from rust_katago_b200 import synthetic

        return synthetic.B11C768_MXFP8

    def gemm_launcher(self, m, n, k, epi, act):
        """A launch of the MXFP8 GEMM on quantised random operands of the given shape."""
        from rust_katago_b200 import _capi, mxfp8

        torch = self.torch
        x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
        _, _, data, scale = mxfp8.dimensions(m, k)
        q = torch.empty(data, dtype=torch.uint8, device="cuda")
        sc = torch.zeros(scale, dtype=torch.uint8, device="cuda")
        st = torch.zeros(2, dtype=torch.int32, device="cuda")
        mxfp8.reset_status(st)
        mxfp8.quantize(x, _capi.DT_BF16, m, k, k, q, sc, st)
        w = mxfp8.Mxfp8Weight(np.random.default_rng(n + k).standard_normal((n, k), np.float32) * 0.02, n, k, k)
        bias = torch.rand(n, device="cuda") * 0.01
        out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
        kind = mxfp8.OUT_BF16_RESIDUAL if epi == _capi.EPI_RES16 else mxfp8.OUT_BF16

        def launch():
            mxfp8.gemm(q, sc, m, w, out, n, kind, st, bias=bias, act=act)

        launch.keep = (x, q, sc, st, w, bias, out)
        return launch


WORKLOADS = {"ffn": FfnWorkload, "trunk": TrunkWorkload, "trunk_mxfp8": TrunkMxfp8Workload}


# ------------------------------------------------------------------ runners
def run_reference(args):
    """CPU arm: the oracle restatement of the reference's quantized CPU path,
    rank 0 only, all host threads, a bounded sample of positions per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle

    oracle.build()
    # explicit: torchrun sets OMP_NUM_THREADS=1 in every rank's environment
    threads = oracle.set_threads(max(1, os.cpu_count() or 1))
    wl = WORKLOADS[args.workload](args.batch, None, seed=1234, build_device=False)
    positions = args.ref_positions
    for _ in range(min(args.warmup, 1)):
        wl.cpu_reference(positions, threads)
    times = [wl.cpu_reference(positions, threads) for _ in range(args.steps)]
    sec = statistics.mean(times)
    value = positions / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": wl.name, "batch_per_gpu": args.batch, "sample_positions_per_step": positions},
        "cpu_baseline": {"value": value, "unit": "positions/s", "cores": threads, "kind": "port",
                         "sample": f"{positions} position(s) ({positions * 361} tokens) of the same workload per "
                                   "step through the CPU oracle (restatement of the reference's W8A8 CPU arithmetic; "
                                   "the Rust reference cannot be built in this image)"},
        "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload == "trunk":
        line["cpu_baseline"]["gemm_config1"] = config1_gemm_record(None, None, threads, gpu=False)
    print(json.dumps(line), flush=True)
    return 0


def time_launches(torch, stream, fn, flush, n):
    """Device times (ms) of fn() over n launches, CUDA events on `stream`,
    with an L2 flush (on the same stream) before each launch outside the events."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for s, e in evs:
        with torch.cuda.stream(stream):
            flush.fill_(1)
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


# ------------------------------------------------------------------ sub-records of the default run
def config1_gemm_record(torch, flush, threads_all, gpu=True):
    """BASELINE config 1 (the reference's CPU W8A8 projection, int8_kernels.rs:273-301,
    bench_lowprec.rs:689-704): A N(0,1) [2888, 768] per-token absmax int8, W N(0,0.02)
    [3072, 768] per-channel int8, int32 dot, dequant to a 16-bit output, in GOP/s:
    the CPU oracle single-threaded and on all host threads (bounded row samples),
    and the same projection on this GPU (kb_int8_project_half)."""
    import oracle

    m, n, k = 2888, 3072, 768
    seed = 0x123456789ABCDEF0 ^ (m * 131 + n * 7 + k)
    rng = np.random.default_rng(seed & 0xFFFFFFFFFFFFFFFF)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    a16 = oracle.f16_encode(a)
    wq, ws = oracle.quantize_weights(w)
    rec = {"shape": [m, n, k], "ops_per_row": 2 * n * k}
    for label, threads, rows in (("cpu_1_thread", 1, 96), ("cpu_all_threads", threads_all, m)):
        oracle.w8a8_project_half(a16[:8], wq, ws, threads=threads)  # warm
        t0 = time.perf_counter()
        oracle.w8a8_project_half(a16[:rows], wq, ws, threads=threads)
        sec = time.perf_counter() - t0
        rec[label] = {"gops": 2.0 * rows * n * k / sec / 1e9, "threads": threads, "rows_sampled": rows}
    if not gpu:
        return rec
    from rust_katago_b200 import int8

    wt = int8.Int8Weight(w)
    wsp = int8.Int8Workspace(m, k, n)
    x = torch.from_numpy(a16.view(np.int16)).cuda()
    out = torch.empty((m, n), dtype=torch.int16, device="cuda")
    stream = torch.cuda.current_stream()  # the workspace's stream

    def launch():
        wsp.project_half(x, k, wt, out, m)

    for _ in range(3):
        launch()
    ms = statistics.mean(time_launches(torch, stream, launch, flush, 10))
    rec["gpu"] = {"gops": 2.0 * m * n * k / (ms / 1e3) / 1e9, "ms": ms,
                  "how": "kb_int8_project_half: quantise fp16 rows, tcgen05 INT8 GEMM, fp16 dequant epilogue"}
    rec["gpu_over_cpu_all_threads"] = rec["gpu"]["gops"] / rec["cpu_all_threads"]["gops"]
    return rec


def handle_forward_ms(torch, handle, batch, d_sp, d_gl, d_out, flush, steps):
    """Device ms per forward (the handle's CUDA graph for `batch`), L2 flushed between."""
    stream = torch.cuda.ExternalStream(handle.stream)
    fwd = lambda: handle.forward_device(batch, d_sp, d_gl, d_out, use_graph=True)  # noqa: E731
    for _ in range(3):
        fwd()
    torch.cuda.synchronize()
    return time_launches(torch, stream, fwd, flush, steps)


def pipelined_rows(handle, spatial, glob, rows, steps):
    """`steps` batches through submit_rows / finish_rows with both pipeline slots in use."""
    tok = handle.submit_rows(spatial, glob, rows)
    for _ in range(steps - 1):
        nxt = handle.submit_rows(spatial, glob, rows)
        handle.finish_rows(tok)
        tok = nxt
    handle.finish_rows(tok)


def trunk_sub_records(wl, torch, flush, steps, world, rank, max_over_ranks, barrier):
    """config5 (1024 positions per GPU) and latency (B = 1, 16) on every rank, max over ranks."""
    from rust_katago_b200 import backend, synthetic

    out = {}
    b5 = 1024
    sp, gl = synthetic.make_positions(b5, 4321 + 7919 * rank)
    h5 = backend.CudaBackend.create_compute_handle(wl.model, b5)
    h5.warmup([b5])
    d_sp, d_gl = torch.from_numpy(sp).cuda(), torch.from_numpy(gl).cuda()
    d_out = torch.zeros(b5 * backend.OUT_PER_POS, device="cuda")
    k5 = max(3, min(steps, 10))
    ms = max_over_ranks(sum(handle_forward_ms(torch, h5, b5, d_sp, d_gl, d_out, flush, k5)))
    rows = backend.row_params(b5, symmetry=np.random.default_rng(rank).integers(0, 8, b5))
    pipelined_rows(h5, sp, gl, rows, 2)
    barrier()
    t0 = time.perf_counter()
    pipelined_rows(h5, sp, gl, rows, k5)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    out["config5"] = {
        "workload": "config5: b11c768 W8A8 trunk, 1024 positions per GPU, batch-sharded, weights replicated",
        "batch_per_gpu": b5, "steps": k5, "ms_per_step": ms / k5,
        "value": b5 * world * k5 / (ms / 1e3), "unit": "positions/s",
        "e2e": {"value": b5 * world * k5 / e2e_s, "unit": "positions/s",
                "how": "kb_submit_rows / kb_finish_rows, two batches in flight, host clock, max over ranks"}}
    del h5, d_sp, d_gl, d_out
    torch.cuda.empty_cache()

    lat = {}
    hl = backend.CudaBackend.create_compute_handle(wl.model, 16)
    hl.warmup([1, 16])
    for b in (1, 16):
        spb, glb = synthetic.make_positions(max(b, 4), 99 + rank)
        spb, glb = spb[:b], glb[:b]
        d_sp, d_gl = torch.from_numpy(spb).cuda(), torch.from_numpy(glb).cuda()
        d_out = torch.zeros(b * backend.OUT_PER_POS, device="cuda")
        dev = handle_forward_ms(torch, hl, b, d_sp, d_gl, d_out, flush, 20)
        rowsb = backend.row_params(b)
        for _ in range(3):
            hl.finish_rows(hl.submit_rows(spb, glb, rowsb))
        rt = []
        for _ in range(30):
            t0 = time.perf_counter()
            hl.finish_rows(hl.submit_rows(spb, glb, rowsb))
            rt.append(time.perf_counter() - t0)
        barrier()
        t0 = time.perf_counter()
        pipelined_rows(hl, spb, glb, rowsb, 30)
        two_s = max_over_ranks(time.perf_counter() - t0)
        lat[f"B{b}"] = {"forward_ms": max_over_ranks(statistics.median(dev)),
                        "e2e_round_trip_ms": max_over_ranks(statistics.median(rt) * 1e3),
                        "e2e_two_in_flight_positions_per_s": b * world * 30 / two_s}
    lat["how"] = ("forward_ms: device time of one graph-launched forward (CUDA events, L2 flushed before); "
                  "e2e_round_trip_ms: host clock of kb_submit_rows -> kb_finish_rows for one batch (median of 30); "
                  "two_in_flight: 30 batches with both pipeline slots in use")
    out["latency"] = lat
    del hl

    # The reference's own TF3 b11c768 topology (nested bottleneck, 11 x 3
    # attention / SwiGLU pairs at width 384, 12 x 32 heads), same batch, both
    # its INT8 recipes: every projection INT8, and the default FFN scope
    # (attention projections binary16).
    tf3 = {}
    sp, gl = synthetic.make_positions(wl.batch, 77 + rank)
    d_sp, d_gl = torch.from_numpy(sp).cuda(), torch.from_numpy(gl).cuda()
    d_out = torch.zeros(wl.batch * backend.OUT_PER_POS, device="cuda")
    for label, topo in (("int8", synthetic.TF3_B11C768), ("ffn_scope", synthetic.TF3_B11C768_FFN)):
        model = backend.CudaBackend.load_model(topo, synthetic.make_blob(topo, 1234), torch.cuda.current_device())
        ht = backend.CudaBackend.create_compute_handle(model, wl.batch)
        ht.warmup([wl.batch])
        kt = max(3, min(steps, 10))
        ms = max_over_ranks(sum(handle_forward_ms(torch, ht, wl.batch, d_sp, d_gl, d_out, flush, kt)))
        tf3[label] = {"ms_per_step": ms / kt, "value": wl.batch * world * kt / (ms / 1e3), "unit": "positions/s"}
        del ht, model
    tf3["workload"] = ("the reference's TF3 b11c768 (nested: C 768, mid 384, 11 x 3 pairs, 12 x 32 heads, SwiGLU "
                       f"1152), batch {wl.batch} per GPU, device time per graph-launched forward")
    out["tf3_b11c768"] = tf3
    return out


def sharded_record(torch, wl, world, steps):
    """One process, one host thread and one compute handle per GPU (the
    reference's evaluator shape, eval.rs:245-330; rust_katago_b200.sharding),
    1024 positions per GPU, decoded rows through kb_submit_rows / kb_finish_rows
    with both pipeline slots in use; host clock around all threads.  Run on
    devices [0] and then [0 .. world-1]."""
    from rust_katago_b200 import backend, sharding, synthetic

    per = 1024
    res = {}
    for devs in ([0], list(range(world))) if world > 1 else ([0],):
        ev = sharding.ShardedEvaluator(wl.topo, wl.blob, devs, per)
        n = per * len(devs)
        sp, gl = synthetic.make_positions(n, 2468)
        rows = backend.row_params(per, symmetry=np.random.default_rng(5).integers(0, 8, per))
        shards = sharding.split_batch(sp, gl, len(devs))
        for i, h in enumerate(ev.handles):
            with torch.cuda.device(devs[i]):
                h.warmup([per])
        k = max(3, min(steps, 10))

        def run(nsteps):
            errs = []

            def work(i):
                try:
                    with torch.cuda.device(devs[i]):
                        _, _, s_i, g_i = shards[i]
                        pipelined_rows(ev.handles[i], s_i, g_i, rows, nsteps)
                except Exception as e:  # surfaced after join
                    errs.append(e)

            ts = [threading.Thread(target=work, args=(i,)) for i in range(len(devs))]
            t0 = time.perf_counter()
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            if errs:
                raise errs[0]
            return time.perf_counter() - t0

        run(2)
        sec = run(k)
        res[len(devs)] = n * k / sec
        del ev
    value = res[max(res)]
    return {"value": value, "unit": "positions/s", "devices": max(res), "positions_per_gpu": per,
            "single_device_value": res[1], "efficiency_vs_n_x_single": value / (max(res) * res[1]),
            "how": "one process, ShardedEvaluator (one handle and host thread per GPU), kb_submit_rows / "
                   "kb_finish_rows with two batches in flight per GPU, pinned staging and H2D/D2H included, "
                   "host clock around all threads"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="trunk")
    ap.add_argument("--batch", type=int, default=None, help="positions per GPU (trunk / trunk_mxfp8 256, ffn 64)")
    ap.add_argument("--ref-positions", type=int, default=1, help="positions per CPU reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config5 / latency / sharded sub-records")
    args = ap.parse_args()
    if args.batch is None:
        args.batch = 64 if args.workload == "ffn" else 256
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from rust_katago_b200 import _capi

    _capi.call("kb_device_check", local)
    wl = WORKLOADS[args.workload](args.batch, torch, seed=1234, **({"rank": rank} if args.workload != "ffn" else {}))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = wl.stream

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        wl.step()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    step_ms = time_launches(torch, stream, wl.step, flush, args.steps)
    barrier()
    clocks = sampler.stop()
    total_ms = max_over_ranks(sum(step_ms))
    ms_per_step = total_ms / args.steps
    value = wl.units_per_step * world * args.steps / (total_ms / 1e3)

    # end to end through the public API with host buffers (host clock, max over ranks)
    wl.e2e_run(2)
    barrier()
    t0 = time.perf_counter()
    wl.e2e_run(args.steps)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = wl.units_per_step * world * args.steps / e2e_s
    h2d, d2h = wl.e2e_bytes()

    # INT8 GEMMs of the step, each timed alone on this stream (same shapes)
    peaks = load_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    gemm_rows = []
    for label, m, n, k, epi, act, per_step in wl.gemms():
        fn = wl.gemm_launcher(m, n, k, epi, act) if hasattr(wl, "gemm_launcher") else gemm_launcher(torch, m, n, k, epi, act)
        for _ in range(3):
            fn()
        ms = statistics.mean(time_launches(torch, torch.cuda.current_stream(), fn, flush, 10))
        gemm_rows.append({"gemm": label, "m": m, "n": n, "k": k, "ms": ms, "per_step": per_step,
                          "tops": 2.0 * m * n * k / (ms / 1e3) / 1e12})
    dom = max(gemm_rows, key=lambda r: r["ms"] * r["per_step"])
    tot_ops = sum(2.0 * r["m"] * r["n"] * r["k"] * r["per_step"] for r in gemm_rows)
    tot_ms = sum(r["ms"] * r["per_step"] for r in gemm_rows)
    traffic = profile_traffic(dom["gemm"])
    roofline = {"bound": "tensor", "achieved": dom["tops"], "peak": int8_peak, "unit": "TFLOP/s",
                "frac": dom["tops"] / int8_peak, "traffic": traffic,
                "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of one launch of this GEMM, "
                                "from the ncu capture summarised in profiles/ (same shape, warm launch)",
                "kernel": f"{getattr(wl, 'kernel', 'gemm_kernel<i8,256>')} {dom['gemm']} "
                          f"(m={dom['m']}, n={dom['n']}, k={dom['k']})",
                "kernel_ms": dom["ms"],
                "peak_note": f"{'FP8' if getattr(wl, 'dtype', 'int8') == 'e4m3' else 'INT8'} dense peak = "
                             f"2 x the {peaks['source']} cuBLAS bf16 burst "
                             f"({peaks['bf16_tflops']} TFLOP/s): tcgen05 kind::i8 issues at twice kind::f16"}
    # The trunk's attention, timed the same way: when its share of the step is
    # the largest, it is the dominant kernel and the roofline describes it.
    att = None
    if hasattr(wl, "attention"):
        label, fn, per_step, nbytes, flops = wl.attention()
        for _ in range(3):
            fn()
        ams = statistics.mean(time_launches(torch, torch.cuda.current_stream(), fn, flush, 10))
        t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9) * 1e3
        t_tc = flops / (peaks["bf16_tflops"] * 1e12) * 1e3
        att = {"kernel": label, "ms": ams, "per_step": per_step, "bytes": nbytes, "flops": flops,
               "hbm_gbs": nbytes / (ams / 1e3) / 1e9, "tflops": flops / (ams / 1e3) / 1e12,
               "bound": "hbm" if t_hbm >= t_tc else "tensor"}
        if ams * per_step > dom["ms"] * dom["per_step"]:
            gemm_roofline = roofline
            hbm = att["bound"] == "hbm"
            roofline = {"bound": att["bound"], "achieved": att["hbm_gbs"] if hbm else att["tflops"],
                        "peak": peaks["hbm_gbs"] if hbm else peaks["bf16_tflops"],
                        "unit": "GB/s" if hbm else "TFLOP/s",
                        "frac": (att["hbm_gbs"] / peaks["hbm_gbs"]) if hbm else (att["tflops"] / peaks["bf16_tflops"]),
                        "traffic": profile_traffic("attention"),
                        "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of one launch, from the ncu "
                                        "capture summarised in profiles/attention_b256.md (same shape)",
                        "kernel": f"attention_fa_kernel<64> {label} (batch {wl.batch})", "kernel_ms": ams,
                        "peak_note": f"{peaks['source']} copy bandwidth; the kernel's ideal time is "
                                     f"{max(t_hbm, t_tc) * 1e3:.0f} us ({att['bound']}-bound: "
                                     f"{nbytes / 1e6:.0f} MB read and written, {flops / 1e9:.1f} GFLOP); what "
                                     "sets its pace is the softmax warps' exponentials on the FMA pipe",
                        "dominant_gemm": gemm_roofline}
    roofline.update({"int8_gemms": gemm_rows,
                     "int8_gemm_frac_of_peak": tot_ops / (tot_ms / 1e3) / 1e12 / int8_peak,
                     "int8_gemm_share_of_step": tot_ms / ms_per_step})
    if att is not None:
        roofline["attention"] = att
        roofline["attention_share_of_step"] = att["ms"] * att["per_step"] / ms_per_step

    # sub-records of the default workload (config 5 and latency on every rank)
    extras = {}
    if args.workload == "trunk" and not args.no_extras:
        extras.update(trunk_sub_records(wl, torch, flush, args.steps, world, rank, max_over_ranks, barrier))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        threads = oracle.set_threads(os.cpu_count() or 1)
        positions = 1
        sec = statistics.mean(wl.cpu_reference(positions, threads) for _ in range(2))
        cpu = {"value": positions / sec, "unit": "positions/s", "cores": threads, "kind": "port",
               "sample": f"{positions} position ({positions * 361} tokens) of the same workload through the CPU "
                         "oracle (restatement of the reference's W8A8 CPU arithmetic), mean of 2 runs",
               "gemm_config1": config1_gemm_record(torch, flush, threads)}

    if world > 1:
        # The one-process sharded run uses every rank's GPU from rank 0; the
        # other ranks wait on a host-side (gloo) barrier, so no collective
        # kernel occupies their GPUs meanwhile.
        from datetime import timedelta

        host_group = dist.new_group(backend="gloo", timeout=timedelta(seconds=900))
        dist.barrier(group=host_group)
        if rank == 0 and args.workload == "trunk" and not args.no_extras:
            extras["sharded_e2e"] = sharded_record(torch, wl, world, args.steps)
        dist.barrier(group=host_group)
        dist.barrier()
        dist.destroy_process_group()
    elif args.workload == "trunk" and not args.no_extras:
        extras["sharded_e2e"] = sharded_record(torch, wl, world, args.steps)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": getattr(wl, "dtype", "int8"),
            "data": "synthetic (seeded: weights N(0,0.02), positions 22 binary planes p=0.3 + 19 N(0,1) globals)",
            "config": {"workload": wl.name, "batch_per_gpu": args.batch, "tokens_per_gpu": args.batch * 361,
                       "parallelism": f"batch-sharded x{world}, weights replicated, no collective",
                       "l2": "256 MiB flush between timed steps (working set also exceeds L2)"},
            "e2e": {"value": e2e_value, "unit": "positions/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "how": wl.e2e_how + ", host clock around the steps, max over ranks"},
            "gpu_launches": wl.launches_per_step * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
