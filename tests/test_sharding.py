"""Host-side multi-GPU logic on CPU: contiguous batch shards, max-over-ranks
timing and reassembly of per-rank outputs, run as two gloo ranks (no GPU).
The per-position evaluator stand-in is the CPU oracle trunk on a tiny
topology: positions are independent, so evaluating shards on separate ranks
and concatenating them must reproduce the single-process batch (to float64
summation-order noise: numpy's BLAS blocks the batched products differently)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rust_katago_b200 import sharding, synthetic

TINY = (64, 1, 2, 32, 128)


def test_shard_bounds_tile_the_batch():
    for total in (0, 1, 7, 256, 1000, 1024):
        for world in (1, 2, 3, 4, 8):
            spans = [sharding.shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_bounds(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle.trunk as ot

        topo = synthetic.Topology(*TINY)
        blob = synthetic.make_blob(topo, 3)
        spatial, glob = synthetic.make_positions(5, 9)
        lo, hi = sharding.shard_bounds(5, world, rank)
        mine = ot.forward(blob, TINY, spatial[lo:hi], glob[lo:hi])
        parts = [None] * world
        dist.all_gather_object(parts, (lo, hi, mine["policy"], mine["value"]))
        slowest = sharding.max_over_ranks(0.25 * (rank + 1), dist)
        if rank == 0:
            np.savez(os.path.join(out_dir, "gathered.npz"),
                     policy=np.concatenate([p[2] for p in parts]), value=np.concatenate([p[3] for p in parts]),
                     bounds=np.array([(p[0], p[1]) for p in parts]), slowest=slowest)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_batch(tmp_path):
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    got = np.load(tmp_path / "gathered.npz")
    import oracle.trunk as ot

    topo = synthetic.Topology(*TINY)
    spatial, glob = synthetic.make_positions(5, 9)
    full = ot.forward(synthetic.make_blob(topo, 3), TINY, spatial, glob)
    assert got["bounds"].tolist() == [[0, 3], [3, 5]]
    np.testing.assert_allclose(got["policy"], full["policy"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(got["value"], full["value"], rtol=1e-9, atol=1e-12)
    assert float(got["slowest"]) == 0.5


@pytest.mark.gpu
def test_sharded_evaluator_threads_match_one_handle(cuda):
    """Two handles (on device 0 twice when only one GPU is visible) driven by
    two host threads return exactly what one handle returns for the batch."""
    n_dev = cuda.cuda.device_count()
    devices = [0, 1] if n_dev > 1 else [0, 0]
    topo = synthetic.B11C768
    blob = synthetic.make_blob(topo, 1234)
    spatial, glob = synthetic.make_positions(7, 31)
    ev = sharding.ShardedEvaluator(topo, blob, devices, 4)
    got = ev.get_output(spatial, glob)
    from rust_katago_b200 import backend

    one = backend.CudaBackend.create_compute_handle(backend.CudaBackend.load_model(topo, blob, 0), 7)
    ref = one.get_output(spatial, glob)
    for f in ("policy", "value", "misc", "moremisc", "ownership"):
        assert np.array_equal(getattr(got, f), getattr(ref, f)), f
