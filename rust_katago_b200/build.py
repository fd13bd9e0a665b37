"""Build the sm_100a shared library ``libkatab200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for ``sm_100a`` only (no other
architecture, no PTX fallback) into ``_build/*.o`` and linked into
``rust_katago_b200/libkatab200.so``.  The library depends on the CUDA runtime
(linked statically by nvcc) and reaches the driver API through
``cudaGetDriverEntryPoint``, so it needs no libcuda at link time.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG.parent / "_build"
LIB = PKG / "libkatab200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
    # host code rounds every multiply and add on its own (the model-file
    # loader folds batch norms with the reference's f32 arithmetic)
    "-Xcompiler",
    "-ffp-contract=off",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA 12.9 toolkit is required to build libkatab200")


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(
        [src.stat().st_mtime]
        + [p.stat().st_mtime for pat in ("*.h", "*.cuh") for p in CSRC.glob(pat)]
        + [p.stat().st_mtime for p in (PKG.parent / "include").glob("*.h")]
    ):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout + res.stderr, flush=True)
    return obj


def build(verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    if LIB.exists() and LIB.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-lz", "-lrt", "-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
