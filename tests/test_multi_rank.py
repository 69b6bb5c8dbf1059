"""Multi-rank host logic on CPU: world_size-2 gloo process groups on 127.0.0.1.

The GPU job runs one engine per rank over a contiguous shard of the streams and reduces
only the timed region's device time (max over ranks); these tests check that plumbing
(sharding, seeds, the max reduction and the job rate) across real processes.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sarbon_b200.multi import job_rate, max_over_ranks, shard_streams, stream_seed


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_streams, times, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        shard = shard_streams(n_streams, world, rank)
        ids = torch.full((n_streams,), -1, dtype=torch.int64)
        ids[list(shard)] = rank
        dist.all_reduce(ids, op=dist.ReduceOp.MAX)       # owner of every stream
        seeds = torch.tensor([stream_seed(0, shard.start)], dtype=torch.int64)
        all_seeds = [torch.zeros_like(seeds) for _ in range(world)]
        dist.all_gather(all_seeds, seeds)
        ms_max = max_over_ranks(times[rank])
        out[rank] = (ids.tolist(), [int(t.item()) for t in all_seeds], ms_max,
                     job_rate(world, len(shard), 100, ms_max))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_streams", [16, 7])
def test_two_rank_sharding_and_timing(n_streams):
    world, port = 2, _free_port()
    times = [12.5, 20.0]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, n_streams, times, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        codes = [p.exitcode for p in procs]
        res = dict(out)
    assert codes == [0, 0], codes
    per = -(-n_streams // world)
    for r in range(world):
        owners, seeds, ms_max, rate = res[r]
        # every stream has exactly one owner, contiguous blocks in rank order
        assert owners == [i // per for i in range(n_streams)]
        assert len(set(seeds)) == world                  # distinct camera content per rank
        assert ms_max == max(times)                      # the job takes the slowest rank's time
        assert rate == pytest.approx(world * len(shard_streams(n_streams, world, r)) * 100 / (max(times) * 1e-3))


def test_shard_edges():
    assert list(shard_streams(0, 2, 1)) == []
    assert [len(shard_streams(5, 8, r)) for r in range(8)] == [1, 1, 1, 1, 1, 0, 0, 0]
    assert sum(len(shard_streams(64, 8, r)) for r in range(8)) == 64
    with pytest.raises(ValueError):
        shard_streams(4, 2, 2)
    assert max_over_ranks(3.0) == 3.0                    # no process group: identity
    with pytest.raises(ValueError):
        job_rate(1, 1, 1, 0.0)
