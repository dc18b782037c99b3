"""The N > 1 host path on the CPU: two `gloo` ranks in separate processes
exercise the sequence sharding, the slowest-rank time and the gathering the
multi-GPU bench and chains use (onnx_runtime_dart_b200/sharding.py)."""
import os
import socket

import numpy as np
import pytest

from onnx_runtime_dart_b200 import sharding


@pytest.mark.parametrize("total", [0, 1, 7, 32, 64, 65])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_the_batch_once(total, world):
    seen = []
    for r in range(world):
        s, c = sharding.shard(total, world, r)
        seen.extend(range(s, s + c))
    assert seen == list(range(total))
    counts = [sharding.shard(total, world, r)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_shard_rejects_bad_arguments():
    with pytest.raises(ValueError):
        sharding.shard(8, 0, 0)
    with pytest.raises(ValueError):
        sharding.shard(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(0)
        prompt = rng.integers(0, 151936, (64, 16)).astype(np.int64)  # the global batch, same on every rank
        mine = sharding.local_slice(prompt, world, rank)
        # A per-sequence computation on the local rows (a stand-in for the chain).
        local_out = mine.sum(axis=1, keepdims=True) % 9973
        gathered = sharding.gather_slices(local_out, dist)
        slowest = sharding.max_over_ranks(10.0 + rank, dist)
        tput = sharding.job_throughput(len(mine) * 16, world, slowest)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"),
                np.array([len(mine), slowest, tput, int(np.array_equal(gathered, prompt.sum(axis=1, keepdims=True) % 9973))],
                         dtype=np.float64))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_time_and_gather(tmp_path):
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    for r, (n, slowest, tput, ok) in enumerate(res):
        assert n == 32
        assert slowest == 11.0          # the slowest rank's time reaches every rank
        assert tput == pytest.approx(64 * 16 / 0.011)
        assert ok == 1                  # the gathered slices rebuild the global batch in order
    del torch
