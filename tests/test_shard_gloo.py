"""Multi-rank host logic on CPU: (batch x head) sharding with 2 gloo ranks.

Each rank computes its contiguous block of flattened heads with the CPU
oracle (standing in for the GPU kernel), times itself, and the ranks agree on
the max time with the same helper bench.py uses; gathering the shards must
reproduce the single-process result exactly."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tda_b200.shard import shard_range


def test_shard_range_partitions():
    for total in (1, 7, 16, 256):
        for world in (1, 2, 3, 4, 8):
            if world > total:
                continue
            shards = [shard_range(total, world, r) for r in range(world)]
            assert shards[0].start == 0 and shards[-1].stop == total
            assert all(a.stop == b.start for a, b in zip(shards, shards[1:]))
            sizes = [s.size for s in shards]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import time

    import torch
    import torch.distributed as dist

    from oracle import tda_oracle as O
    from tda_b200.shard import max_over_ranks, shard_range, sum_over_ranks
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, H, S, D = 2, 3, 40, 16
    rng = np.random.default_rng(0)
    xs = [rng.standard_normal((B, H, S, D)) for _ in range(5)]
    sh = shard_range(B * H, world, rank)
    flat = [x.reshape(1, B * H, S, D)[:, sh.start:sh.stop] for x in xs]
    t0 = time.perf_counter()
    part = O.diff_fwd(*flat, 1.0, 0.5, 2.0, True)
    dt = time.perf_counter() - t0
    tmax = max_over_ranks(dt)
    assert tmax >= dt
    assert sum_over_ranks(sh.size) == B * H
    np.save(os.path.join(out_dir, f"part{rank}.npy"), part)
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_reproduce_single_process(tmp_path):
    from oracle import tda_oracle as O
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    parts = [np.load(tmp_path / f"part{r}.npy") for r in range(world)]
    got = np.concatenate(parts, axis=1).reshape(2, 3, 40, 16)
    rng = np.random.default_rng(0)
    xs = [rng.standard_normal((2, 3, 40, 16)) for _ in range(5)]
    want = O.diff_fwd(*xs, 1.0, 0.5, 2.0, True)
    np.testing.assert_array_equal(got, want)
