"""Batch sharding of independent board positions over the GPUs of one box.

Positions never interact in the trunk (attention stays inside one board's 361
tokens), so a batch splits into contiguous per-GPU shards with the weights
replicated on every device and no collective on the data path.  Two ways to
drive it:

* one process per GPU (``torchrun``; ``bench.py`` does this): rank r evaluates
  ``shard_bounds(total, world, r)`` of the global batch on ``cuda:r``; the only
  cross-rank traffic is host-side bookkeeping (barriers, the max-over-ranks
  timing, an optional gather of outputs);
* one process, one thread and one compute handle per GPU
  (:class:`ShardedEvaluator`), the shape of the reference's evaluator, whose
  server threads each own a handle bound to ``gpu_idx_for_this_thread``
  (crates/kata_nn/src/eval.rs:245-330, backend.rs:206-410).
"""

from __future__ import annotations

import threading

import numpy as np


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) of `total` positions owned by `rank` of `world`;
    shard sizes differ by at most one and the shards tile [0, total)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("need world > 0, 0 <= rank < world, total >= 0")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, dist=None, device: str = "cpu") -> float:
    """Max of a per-rank float over the process group (the time of the slowest
    rank); the value itself when no group is initialised."""
    if dist is None or not dist.is_available() or not dist.is_initialized():
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def split_batch(spatial: np.ndarray, glob: np.ndarray, world: int):
    """[(lo, hi, spatial[lo:hi], glob[lo:hi])] for every rank (empty shards kept)."""
    n = spatial.shape[0]
    out = []
    for r in range(world):
        lo, hi = shard_bounds(n, world, r)
        out.append((lo, hi, spatial[lo:hi], glob[lo:hi]))
    return out


def concat_outputs(parts):
    """Concatenate per-shard NNOutputs (in rank order) into one NNOutputs."""
    from .backend import NNOutputs

    parts = [p for p in parts if p is not None and p.policy.shape[0] > 0]
    return NNOutputs(*(np.concatenate([getattr(p, f) for p in parts], axis=0)
                       for f in ("policy", "value", "misc", "moremisc", "ownership")))


class ShardedEvaluator:
    """One model copy and one compute handle per device; get_output splits the
    batch contiguously and evaluates the shards concurrently, one host thread
    per device (each ctypes call releases the GIL)."""

    def __init__(self, topology, blob: np.ndarray, devices, max_batch_per_device: int):
        from .backend import CudaBackend

        self.devices = list(devices)
        self.max_batch = max_batch_per_device
        self.models = [CudaBackend.load_model(topology, blob, d) for d in self.devices]
        self.handles = [CudaBackend.create_compute_handle(m, max_batch_per_device) for m in self.models]

    def get_output(self, spatial: np.ndarray, glob: np.ndarray, symmetry=None):
        shards = split_batch(spatial, glob, len(self.devices))
        syms = [None if symmetry is None else np.asarray(symmetry, np.int32)[lo:hi] for lo, hi, _, _ in shards]
        if max(hi - lo for lo, hi, _, _ in shards) > self.max_batch:
            raise ValueError("batch exceeds devices x max_batch_per_device")
        results: list = [None] * len(shards)
        errors: list = []

        def work(i, sp, gl):
            try:
                if sp.shape[0] > 0:
                    results[i] = self.handles[i].get_output(sp, gl, syms[i])
            except Exception as e:  # re-raised on the calling thread
                errors.append(e)

        threads = [threading.Thread(target=work, args=(i, sp, gl)) for i, (_, _, sp, gl) in enumerate(shards)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        return concat_outputs(results)
