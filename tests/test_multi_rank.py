"""The benchmark's multi-rank host logic on CPU ranks (gloo, world size 2): every rank takes a
disjoint contiguous shard of the seeded global batch, the shards cover it, and every rank
reads back the maximum of the per-rank step times."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lo, hi = bench.shard_bounds(8, world, rank)
        rng = np.random.default_rng(bench.DATA_SEED)
        x_all = rng.normal(size=(8, 3, 4, 4)).astype(np.float32)
        shard = x_all[lo:hi]
        step_ms = 1.0 + rank * 0.5  # rank 1 is the slower one
        got = bench.reduce_max(step_ms, world)
        np.save(os.path.join(out_dir, f"shard{rank}.npy"), shard)
        with open(os.path.join(out_dir, f"max{rank}.txt"), "w") as f:
            f.write(repr(got))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    import bench
    rng = np.random.default_rng(bench.DATA_SEED)
    x_all = rng.normal(size=(8, 3, 4, 4)).astype(np.float32)
    shards = [np.load(tmp_path / f"shard{r}.npy") for r in range(world)]
    np.testing.assert_array_equal(np.concatenate(shards), x_all)
    for r in range(world):
        assert float((tmp_path / f"max{r}.txt").read_text()) == 1.5


def test_shard_bounds_rejects_uneven_split():
    import bench
    assert bench.shard_bounds(256, 8, 7) == (224, 256)
    with pytest.raises(ValueError):
        bench.shard_bounds(10, 4, 0)
