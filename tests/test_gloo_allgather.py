"""Fitness all-gather (the one collective) on world-size-2 gloo ranks, CPU."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, sizes, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from zerograd_b200 import allgather_losses, compute_partition_sizes
        from zerograd_b200._distributed import shard_ranges

        a, b = shard_ranges(sizes)[rank]
        local = torch.arange(a, b, dtype=torch.float32) * 10.0
        full = allgather_losses(local, sizes)
        q.put((rank, full.tolist(), compute_partition_sizes(sum(sizes), [1.0] * world)))
    finally:
        dist.destroy_process_group()


def _run(sizes):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, len(sizes), port, sizes, q)) for r in range(len(sizes))]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return sorted(out)


def test_uneven_allgather_is_in_candidate_order():
    out = _run([3, 5])
    expect = [float(i) * 10.0 for i in range(8)]
    for rank, full, _ in out:
        assert full == expect


def test_empty_shard():
    out = _run([0, 4])
    for rank, full, _ in out:
        assert full == [0.0, 10.0, 20.0, 30.0]
