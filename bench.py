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

    def __init__(self, batch: int, torch, seed: int = 1234):
        from rust_katago_b200 import int8

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
        self.resid_h = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        self.up = int8.Int8Weight(self.up_w)
        self.down = int8.Int8Weight(self.down_w)
        self.ws = int8.Int8Workspace(self.rows, self.f, self.f)
        dev = "cuda"
        self.gamma = torch.from_numpy(self.gamma_h).to(dev)
        self.up_b = torch.from_numpy(self.up_b_h).to(dev)
        self.down_b = torch.from_numpy(self.down_b_h).to(dev)
        self.resid = torch.from_numpy(self.resid_h.view(np.int16)).to(dev)
        self.pinned_in = torch.from_numpy(self.resid_h.view(np.int16)).pin_memory()
        self.pinned_out = torch.empty_like(self.pinned_in).pin_memory()
        self.launches_per_step = 4

    @property
    def units_per_step(self):
        return self.batch

    def step(self):
        self.ws.ffn_gelu_rms(self.gamma, 1e-6, self.up, self.up_b, self.down, self.down_b, self.resid, self.rows)

    def e2e_step(self):
        self.resid.copy_(self.pinned_in, non_blocking=True)
        self.step()
        self.pinned_out.copy_(self.resid, non_blocking=True)

    def e2e_bytes(self):
        b = self.rows * self.c * 2
        return b, b

    def dominant(self):
        """(label, launch fn, algorithmic ops per launch) of the dominant kernel."""
        from rust_katago_b200 import _capi, int8

        t = self.torch
        m, n, k = self.rows, self.f, self.up.kp
        a = t.randint(-127, 128, (m, k), dtype=t.int8, device="cuda")
        sa = t.rand(m, device="cuda") * 0.01
        out = t.empty((m, n), dtype=t.bfloat16, device="cuda")
        sw = t.rand(n, device="cuda") * 0.01

        w = _WeightView(self.up)

        def launch():
            int8.linear(a, sa, w, sw, self.up_b, m, n, k, _capi.EPI_16, out, n, act=_capi.ACT_GELU)

        return "gemm_kernel<i8, 256, Epi16> (up projection 768->3072 + bias + GELU)", launch, 2 * m * n * self.c

    def cpu_reference(self, positions: int, threads: int):
        """The CPU oracle on `positions` positions; returns seconds."""
        import oracle

        rows = positions * 361
        t0 = time.perf_counter()
        oracle.gelu_ffn_bf16(np.ascontiguousarray(self.resid_h[:rows]), self.gamma_h, 1e-6, self.up_w, self.up_b_h,
                             self.down_w, self.down_b_h, threads=threads)
        return time.perf_counter() - t0


class _WeightView:
    """Expose an uploaded weight's device pointer to the kernel-level calls."""

    def __init__(self, w):
        self.w = w

    def data_ptr(self):
        return self.w.q_ptr


WORKLOADS = {"ffn": FfnWorkload}


# ------------------------------------------------------------------ runners
def run_reference(args):
    """CPU arm: the oracle restatement of the reference's quantized CPU path."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle

    oracle.build()
    threads = max(1, os.cpu_count() or 1)
    wl_cls = WORKLOADS[args.workload]
    positions = args.ref_positions
    wl = wl_cls.__new__(wl_cls)
    CpuOnly.init(wl, args.batch, positions)
    for _ in range(max(0, min(args.warmup, 1))):
        wl.cpu_reference(positions, threads)
    times = [wl.cpu_reference(positions, threads) for _ in range(args.steps)]
    sec = statistics.mean(times)
    value = positions / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": wl_cls.name, "batch_per_gpu": args.batch, "sample_positions": positions},
        "cpu_baseline": {"value": value, "unit": "positions/s", "cores": threads, "kind": "port",
                         "sample": f"{positions} positions ({positions * 361} tokens) of the same workload per step"},
        "e2e": {"value": value, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


class CpuOnly:
    """Build only the host-side data of a workload (the CPU arm needs no GPU)."""

    @staticmethod
    def init(wl, batch, positions):
        rng = np.random.default_rng(1234)
        wl.batch = batch
        wl.rows = positions * 361
        wl.c, wl.f = 768, 3072
        wl.gamma_h = (1 + 0.02 * rng.standard_normal(wl.c)).astype(np.float32)
        wl.up_w = (0.02 * rng.standard_normal((wl.f, wl.c))).astype(np.float32)
        wl.down_w = (0.02 * rng.standard_normal((wl.c, wl.f))).astype(np.float32)
        wl.up_b_h = (0.02 * rng.standard_normal(wl.f)).astype(np.float32)
        wl.down_b_h = (0.02 * rng.standard_normal(wl.c)).astype(np.float32)
        import oracle

        x = rng.standard_normal((wl.rows, wl.c)).astype(np.float32)
        wl.resid_h = oracle.bf16_encode(x)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="ffn")
    ap.add_argument("--batch", type=int, default=64, help="positions per GPU")
    ap.add_argument("--ref-positions", type=int, default=16, help="positions per CPU sample step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    from rust_katago_b200 import _capi

    _capi.call("kb_device_check", local)
    wl = WORKLOADS[args.workload](args.batch, torch, seed=1234)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        wl.step()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for s, e in events:
        flush.fill_(1)
        s.record(stream)
        wl.step()
        e.record(stream)
    barrier()
    clocks = sampler.stop()
    step_ms = [s.elapsed_time(e) for s, e in events]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = wl.units_per_step * world * args.steps / (total_ms / 1e3)

    # end to end through the public API with host buffers
    for _ in range(2):
        wl.e2e_step()
    barrier()
    e_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for s, e in e_events:
        flush.fill_(1)
        s.record(stream)
        wl.e2e_step()
        e.record(stream)
    barrier()
    e_ms = sum(s.elapsed_time(e) for s, e in e_events)
    te = torch.tensor([e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = wl.units_per_step * world * args.steps / (float(te.item()) / 1e3)
    h2d, d2h = wl.e2e_bytes()

    # dominant kernel, timed alone on the same stream
    label, launch, ops = wl.dominant()
    for _ in range(3):
        launch()
    k_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
    for s, e in k_events:
        flush.fill_(1)
        s.record(stream)
        launch()
        e.record(stream)
    torch.cuda.synchronize()
    k_ms = statistics.mean(s.elapsed_time(e) for s, e in k_events)
    peaks = load_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    achieved = ops / (k_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                "frac": achieved / int8_peak, "traffic": None, "kernel": label,
                "peak_note": f"INT8 dense peak taken as 2x the {peaks['source']} cuBLAS bf16 burst "
                             f"({peaks['bf16_tflops']} TFLOP/s), tcgen05 kind::i8 issuing twice the kind::f16 rate",
                "kernel_ms": k_ms}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        threads = os.cpu_count() or 1
        positions = 2
        wl.cpu_reference(1, threads)
        sec = statistics.mean(wl.cpu_reference(positions, threads) for _ in range(2))
        cpu = {"value": positions / sec, "unit": "positions/s", "cores": threads, "kind": "port",
               "sample": f"{positions} positions ({positions * 361} tokens) of the same workload, CPU oracle"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded N(0,1) residual, N(0,0.02) weights)",
            "config": {"workload": wl.name, "batch_per_gpu": args.batch, "tokens_per_gpu": args.batch * 361,
                       "parallelism": f"batch-sharded x{world}, weights replicated, no collective",
                       "l2": "256 MiB flush between timed steps"},
            "e2e": {"value": e2e_value, "unit": "positions/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": wl.launches_per_step * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
