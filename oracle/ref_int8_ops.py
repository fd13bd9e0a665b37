"""The reference's own INT8 boundary kernels, compiled unmodified, as a
second, GPU-side oracle — TEST INFRASTRUCTURE ONLY.

Rust_KataGo's crates/kata_nn/cuda-kernels/int8_ops.cu is compiled straight
from the reference tree by build() with the flags of the reference's own
build script (-O3 --std=c++17, no fast math: crates/kata_nn/build.rs:700-720)
for sm_100a into oracle/_ref/int8_ops.sm_100a.cubin (ignored by git, carried
with the working tree; nothing of the source is copied).  The cubin is loaded
through the CUDA driver API in the context torch has made current and its
kernels are launched with the reference's launch shapes (int8.rs:890-925,
:1160-1182, :1228-1260; cudarc's LaunchConfig::for_num_elems for the
dequantisers).  They are the reference's exact arithmetic on the GPU: the
fp16 boundaries, the lane-strided RMS sum with rsqrtf, and CUDA's expf in the
SwiGLU.  Only tests/ load this module.
"""

from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
CUBIN = HERE / "_ref" / "int8_ops.sm_100a.cubin"
SOURCE_IN_REFERENCE = Path("crates/kata_nn/cuda-kernels/int8_ops.cu")


def reference_root() -> Path:
    return Path(os.environ.get("KB_REFERENCE_ROOT", "/root/reference"))


def build() -> Path | None:
    """Compile the reference's int8_ops.cu for sm_100a (returns the cubin, or
    None when the reference tree is not present and no cubin was built)."""
    src = reference_root() / SOURCE_IN_REFERENCE
    if not src.exists():
        return CUBIN if CUBIN.exists() else None
    if CUBIN.exists() and CUBIN.stat().st_mtime >= src.stat().st_mtime:
        return CUBIN
    CUBIN.parent.mkdir(exist_ok=True)
    nvcc = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--std=c++17", str(src), "-o",
           str(CUBIN)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for the reference's int8_ops.cu:\n{res.stderr}")
    return CUBIN


class RefKernels:
    """The reference kernels on the current device (needs a current CUDA context)."""

    def __init__(self):
        if not CUBIN.exists():
            raise FileNotFoundError(f"{CUBIN} is missing: run oracle.ref_int8_ops.build() where the reference is")
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.module = ctypes.c_void_p()
        self._check(self.cu.cuModuleLoad(ctypes.byref(self.module), str(CUBIN).encode()), "cuModuleLoad")
        self.funcs = {}

    @staticmethod
    def _check(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed with CUresult {rc}")

    def _func(self, name):
        if name not in self.funcs:
            f = ctypes.c_void_p()
            self._check(self.cu.cuModuleGetFunction(ctypes.byref(f), self.module, name.encode()), name)
            self.funcs[name] = f
        return self.funcs[name]

    def launch(self, name, grid, block, args, smem=0, stream=0):
        """args: ("p", device pointer) | ("i", int) | ("f", float)."""
        holders = []
        for kind, v in args:
            holders.append(ctypes.c_void_p(v) if kind == "p" else ctypes.c_int(v) if kind == "i" else ctypes.c_float(v))
        params = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.pointer(h), ctypes.c_void_p) for h in holders])
        self.cu.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 6 + [ctypes.c_uint, ctypes.c_void_p,
                                                                                    ctypes.c_void_p, ctypes.c_void_p]
        self._check(self.cu.cuLaunchKernel(self._func(name), grid, 1, 1, block, 1, 1, smem, ctypes.c_void_p(stream),
                                           params, None), f"launch {name}")

    # ---- the reference's launch shapes
    def rms_quantize(self, x, gamma, q, scales, eps, rows, width):
        name = {384: "int8_rms_quantize384_kernel", 512: "int8_rms_quantize512_kernel"}[width]
        self.launch(name, (rows + 3) // 4, 128, [("p", x), ("p", gamma), ("p", q), ("p", scales), ("f", eps),
                                                  ("i", rows)])

    def quantize_rows(self, x16, q, scales, rows, width, stride, padded, warp):
        name = "int8_quantize_rows_warp_kernel" if warp else "int8_quantize_rows_kernel"
        self.launch(name, (rows + 3) // 4 if warp else rows, 128 if warp else 256,
                    [("p", x16), ("p", q), ("p", scales), ("i", rows), ("i", width), ("i", stride), ("i", padded)])

    def swiglu_quantize(self, dots, scales, sw, q, rows, hidden, padded, warp):
        name = "int8_swiglu_quantize_warp512_kernel" if warp else "int8_swiglu_quantize_kernel"
        self.launch(name, (rows + 3) // 4 if warp else rows, 128 if warp else 256,
                    [("p", dots), ("p", scales), ("p", sw), ("p", q), ("i", rows), ("i", hidden), ("i", padded)],
                    smem=0 if warp else hidden * 4)

    def dequantize(self, dots, sa, sw, out, rows, cols, residual):
        name = "int8_dequantize_residual_kernel" if residual else "int8_dequantize_half_kernel"
        count = rows * cols
        self.launch(name, (count + 1023) // 1024, 1024, [("p", dots), ("p", sa), ("p", sw), ("p", out), ("i", rows),
                                                         ("i", cols)])
