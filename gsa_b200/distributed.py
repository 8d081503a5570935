# SPDX-License-Identifier: Apache-2.0
"""Scene sharding across ranks (one process per GPU).

Scenes are independent, so the query path shards by scene with no exchange
on the data path: rank r owns its own scenes, builds its own forest and
answers its own queries.  The only collectives are timing (the maximum over
ranks of the device time) and one final gather of every rank's answered-row
count and output checksum.  The functions work with any backend
(``nccl`` on GPUs, ``gloo`` on CPUs).
"""

import torch
import torch.distributed as dist


def world():
    """(rank, world size) of the default process group, (0, 1) without one."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def shard_seeds(rank, world_size, total):
    """Scenes of a rank when ``total`` scenes are split over ``world_size``
    GPUs: scene i goes to rank i mod world_size (strong scaling: the job is
    fixed, each rank gets about total / world_size scenes)."""
    return list(range(rank, total, world_size))


def rank_seeds(rank, scenes_per_rank):
    """Scene seeds of a rank: rank * scenes_per_rank + i (weak scaling)."""
    return [rank * scenes_per_rank + i for i in range(scenes_per_rank)]


def barrier():
    """Wait for every rank (no-op without a process group)."""
    if world()[1] > 1:
        dist.barrier()


def max_over_ranks(value, device="cpu"):
    """Largest value over all ranks (e.g. the slowest rank's device time)."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if world()[1] > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_counts(rows, checksum, device="cpu"):
    """[(rows, checksum)] of every rank, in rank order, on every rank."""
    mine = torch.tensor([int(rows), int(checksum)], dtype=torch.int64, device=device)
    n = world()[1]
    if n == 1:
        return [tuple(mine.tolist())]
    out = [torch.zeros(2, dtype=torch.int64, device=device) for _ in range(n)]
    dist.all_gather(out, mine)
    return [tuple(t.tolist()) for t in out]


def output_checksum(outputs):
    """Sum over all integer ID rows of a hierarchy result (int64, on device)."""
    total = None
    for key, v in outputs.items():
        if key.startswith(("ball", "hit", "nni")):
            s = v.to(torch.int64).sum()
            total = s if total is None else total + s
    return int(total.item()) if total is not None else 0
