"""Multi-GPU plumbing of the engine: camera streams are independent, so a job of S streams
on G GPUs runs one engine per GPU (one process per GPU under torchrun) over a contiguous
shard of the streams, with no collective on the hot path.  Only the job-level timing is
reduced across ranks (the max of the per-rank device times), outside the timed region.

Reference: the reference runs its cameras serially in one process
(sarbon/inference/video.py:205); stream sharding across GPUs is this build's own plan for
the multi-camera configuration (independent streams, per-stream caches resident in HBM).
"""
from __future__ import annotations

import torch


def shard_streams(n_streams: int, world: int, rank: int) -> range:
    """Global ids of the streams rank `rank` of `world` owns: a contiguous block,
    stream i on rank i // ceil(n_streams / world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if n_streams < 0:
        raise ValueError("negative stream count")
    per = -(-n_streams // world)
    lo = min(rank * per, n_streams)
    return range(lo, min(lo + per, n_streams))


def stream_seed(base_seed: int, global_stream: int) -> int:
    """Seed of one camera stream's synthetic content: distinct for every global stream id,
    so no two ranks generate the same camera."""
    return 1 + base_seed + 1000 * global_stream


def max_over_ranks(value: float, device=None) -> float:
    """All-reduce MAX of a per-rank float (e.g. the device time of the timed region) over
    the default process group; the identity without one."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_rate(world: int, streams_per_rank: int, steps: int, ms_max: float) -> float:
    """Whole-job frames/s: every rank processed streams_per_rank frames per step for
    `steps` steps; the job took the slowest rank's time."""
    if ms_max <= 0:
        raise ValueError("non-positive time")
    return world * streams_per_rank * steps / (ms_max * 1e-3)
