"""The multi-rank host logic of bench.py on CPU (two gloo ranks): every rank builds its own
shard of the global batch (together they are the single-rank batch, pair for pair), the
timing is the maximum over the ranks, and the host-side barrier around rank-0-only work
holds the other rank until rank 0 is done."""

from __future__ import annotations

import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
HW = (6, 10)
TOTAL = 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench

    first, per = bench.shard_pairs(TOTAL, world, rank)
    img1, img2 = bench.make_inputs(first, per, HW)
    np.savez(os.path.join(out_dir, f"shard{rank}.npz"), first=first, img1=img1, img2=img2)
    # max over ranks
    got = bench.all_max(dist, 0.5 + rank)
    # host-side barrier around rank-0-only work: rank 1 must not pass before rank 0 is done
    host = dist.new_group(backend="gloo")
    dist.barrier(group=host)
    t_done = 0.0
    if rank == 0:
        time.sleep(0.5)
        t_done = time.time()
    dist.barrier(group=host)
    t_pass = time.time()
    np.savez(os.path.join(out_dir, f"sync{rank}.npz"), got=got, t_done=t_done, t_pass=t_pass)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_shard_reduce_and_wait(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    sys.path.insert(0, str(ROOT))
    import bench

    full1, full2 = bench.make_inputs(0, TOTAL, HW)
    shards = [np.load(tmp_path / f"shard{r}.npz") for r in range(world)]
    assert [int(s["first"]) for s in shards] == [0, TOTAL // world]
    np.testing.assert_array_equal(np.concatenate([s["img1"] for s in shards]), full1)
    np.testing.assert_array_equal(np.concatenate([s["img2"] for s in shards]), full2)
    sync = [np.load(tmp_path / f"sync{r}.npz") for r in range(world)]
    assert all(float(s["got"]) == 1.5 for s in sync)
    assert float(sync[1]["t_pass"]) >= float(sync[0]["t_done"])


def test_shard_pairs_rejects_uneven_batches():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.shard_pairs(64, 8, 3) == (24, 8)
    with pytest.raises(AssertionError):
        bench.shard_pairs(64, 3, 0)
