# SPDX-License-Identifier: Apache-2.0
"""CPU: the multi-rank path with two gloo ranks.

Five scenes are split over two ranks (scene i to rank i mod 2); each rank
answers the radius + 3NN hierarchy of its own scenes with the CPU
oracle standing in for the GPU engine (the host logic is what is tested:
scene sharding, max-over-ranks timing, the final gather of row counts and
checksums), and every rank must see the same gathered table.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from gsa_b200 import distributed as gd, scenes
        from oracle import numpy_oracle as orc

        assert gd.world() == (rank, world)
        seeds = gd.shard_seeds(rank, world, 5)
        rows, checksum = 0, 0
        sizes, radii = (400, 100, 25, 6, 1), (0.3, 0.5, 0.9, 1.5)
        for s in seeds:
            p, _ = scenes.room(s, n=sizes[0])
            out, r = orc.hierarchy_oracle(p, sizes, radii)
            rows += r
            checksum += int(sum(v.astype(np.int64).sum() for k, v in out.items() if k.startswith(("ball", "hit", "nni"))))
        slowest = gd.max_over_ranks(10.0 + rank)
        table = gd.gather_counts(rows, checksum)
        q.put((rank, seeds, slowest, table))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_gather():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    (r0, seeds0, slow0, table0), (r1, seeds1, slow1, table1) = results
    assert seeds0 == [0, 2, 4] and seeds1 == [1, 3]
    assert slow0 == slow1 == 11.0
    assert table0 == table1 and len(table0) == 2
    assert table0[0] != table0[1]  # different scenes, different checksums
    assert all(rows > 0 for rows, _ in table0)


def test_single_process_defaults():
    from gsa_b200 import distributed as gd

    assert gd.world() == (0, 1)
    assert gd.rank_seeds(3, 4) == [12, 13, 14, 15]
    assert gd.shard_seeds(0, 1, 3) == [0, 1, 2]
    assert gd.shard_seeds(3, 8, 64) == list(range(3, 64, 8))
    assert sorted(s for r in range(8) for s in gd.shard_seeds(r, 8, 64)) == list(range(64))
    assert gd.max_over_ranks(2.5) == 2.5
    assert gd.gather_counts(7, 9) == [(7, 9)]
    out = {"ball0": torch.tensor([[1, 2]]), "nnd0": torch.tensor([[0.5]]), "nni0": torch.tensor([[3]])}
    assert gd.output_checksum(out) == 6
