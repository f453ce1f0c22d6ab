"""Multi-rank host logic of bench.py on CPU (gloo, world size 2 and 4): the sequence shards tile the
4096-sequence workload exactly once, and the integer outputs gathered to rank 0 keep rank order."""
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
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world)
    s0, ns = bench.shard(rank, world)
    # stand-in per-sequence integer outputs: the global sequence index, as the digests would be
    mine = torch.arange(s0, s0 + ns, dtype=torch.int64)
    parts = [torch.empty(ns, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(parts, mine)
    counts = torch.tensor([ns, 1], dtype=torch.int64)
    dist.all_reduce(counts)
    if rank == 0:
        q.put((torch.cat(parts).numpy().tolist(), counts.tolist()))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_shards_cover_workload_once(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, counts = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == list(range(4096))
    assert counts == [4096, world]
