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


def _leaving_rank_main(rank, world, port, out_dir):
    """Rank 1 runs one step and leaves between steps (no collective of its in flight); rank 0
    finds out at its next collective, which the short process-group timeout bounds."""
    import datetime
    import time

    import torch.distributed as dist

    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    bench.reduce_max(1.0 + rank, world)  # step 0: both ranks
    if rank == 1:
        os._exit(0)  # leaves between steps
    t0 = time.monotonic()
    err = ""
    try:
        bench.reduce_max(1.0, world)  # step 1: the peer is gone
    except Exception as e:  # noqa: BLE001 -- any error is the detection
        err = type(e).__name__ + ": " + str(e)[:200]
    with open(os.path.join(out_dir, "detect0.txt"), "w") as f:
        f.write(f"{time.monotonic() - t0:.3f}\n{err}")
    os._exit(0)


def test_rank_that_leaves_is_detected_at_the_next_collective(tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_leaving_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    elapsed, err = (tmp_path / "detect0.txt").read_text().split("\n", 1)
    assert err, "rank 0's collective returned although its peer had left"
    assert float(elapsed) < 30.0
