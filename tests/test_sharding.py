"""Multi-rank host logic on CPU (gloo, world size 2): the utterance shards of
bench.py (strong scaling: one batch shared out; weak scaling: a batch per
rank) cover every utterance exactly once with no exchange between ranks,
each rank's shard reproduces the single-process result of the oracle on its
utterances, and the timing reductions give the max (time) and the sum (work)
over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shards_partition_every_config(monkeypatch):
    import bench
    monkeypatch.setattr(bench, "SCALING", "strong")
    for n in (1, 5, 32, 64, 160, 320):
        for world in (1, 2, 3, 4, 8):
            got = []
            for r in range(world):
                lo, hi = bench.shard(n, r, world)
                assert 0 <= lo <= hi <= n
                got.extend(range(lo, hi))
            assert got == list(range(n))
            sizes = [bench.shard(n, r, world)[1] - bench.shard(n, r, world)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_weak_scaling_gives_each_rank_a_whole_batch(monkeypatch):
    import bench
    monkeypatch.setattr(bench, "SCALING", "weak")
    for n in (1, 5, 32, 64, 320):
        for world in (1, 2, 4, 8):
            got = []
            for r in range(world):
                lo, hi = bench.shard(n, r, world)
                assert hi - lo == n
                got.extend(range(lo, hi))
            assert got == list(range(n * world))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    from oracle import oracle as O
    bench.SCALING = "strong"
    # A small encoder batch sharded like config 3 under strong scaling.
    batch, t, h = 5, 40, 2
    d = h * 64
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal(batch * t * d).astype(np.float32) for _ in range(3))
    lo, hi = bench.shard(batch, rank, world)
    sl = slice(lo * t * d, hi * t * d)
    out = O.flash_attention_2_batched(q[sl], k[sl], v[sl], hi - lo, t, t, h, d, False, 1)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), out)
    mx = bench.max_over_ranks(float(rank + 1), world)
    tot = bench.sum_over_ranks(float(hi - lo), world)
    np.save(os.path.join(out_dir, f"red{rank}.npy"), np.array([mx, tot]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_shard_without_exchange(tmp_path):
    from oracle import oracle as O
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    parts = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    batch, t, h = 5, 40, 2
    d = h * 64
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal(batch * t * d).astype(np.float32) for _ in range(3))
    full = O.flash_attention_2_batched(q, k, v, batch, t, t, h, d, False, 1)
    assert np.array_equal(np.concatenate(parts), full)
    for r in range(world):
        mx, tot = np.load(tmp_path / f"red{r}.npy")
        assert mx == world and tot == batch
